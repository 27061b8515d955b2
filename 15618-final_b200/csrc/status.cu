// status.cu -- the library's device-side condition word for kernels that run
// without a caller workspace (unpermute, grouped FFN).  Kernels OR
// MOE_B200_DEV_* bits into it instead of trapping; moe_b200_device_status()
// reads and clears it.
#include <mutex>

#include <cuda_runtime.h>

#include "common.cuh"
#include "moe_b200.h"

static __device__ uint32_t g_moe_b200_device_status;

namespace moe_b200 {
int fail(int code, const char* fmt, ...);
int cuda_fail(cudaError_t err, const char* where);

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_mutex;
uint32_t* g_addr[kMaxDevices] = {};
}  // namespace

// Device address of the status word on the current device (looked up once per
// device); nullptr if the lookup fails.
uint32_t* device_status_word() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
    std::lock_guard<std::mutex> lock(g_mutex);
    if (!g_addr[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_moe_b200_device_status) != cudaSuccess) return nullptr;
        g_addr[dev] = static_cast<uint32_t*>(p);
    }
    return g_addr[dev];
}
}  // namespace moe_b200

extern "C" int moe_b200_device_status(void* stream, int* device_status) {
    using namespace moe_b200;
    if (!device_status) return fail(MOE_B200_ERR_INVALID_ARG, "device_status: null output");
    uint32_t* word = device_status_word();
    if (!word) return fail(MOE_B200_ERR_CUDA, "device_status: status word unavailable");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    uint32_t bits = 0;
    cudaError_t err = cudaMemcpyAsync(&bits, word, 4, cudaMemcpyDeviceToHost, s);
    if (err == cudaSuccess) err = cudaStreamSynchronize(s);
    if (err == cudaSuccess && bits) err = cudaMemsetAsync(word, 0, 4, s);
    if (err == cudaSuccess) err = cudaStreamSynchronize(s);
    if (err != cudaSuccess) return cuda_fail(err, "device_status");
    *device_status = int(bits);
    return MOE_B200_OK;
}
