// pack_noalloc.cu -- moe_b200_pack_noalloc: the packing entry point for
// callers that cannot allocate device memory.
//
// Some callers own only their input and output buffers: a plugin running
// inside a host framework that hands out device memory from its own pool and
// forbids direct cudaMalloc, or a thin FFI binding that receives device
// pointers and has no allocator of its own.  moe_b200_pack needs a caller
// workspace; this entry point instead uses scratch memory built into the
// library: a file-scope __device__ array of MOE_B200_NOALLOC_SCRATCH_BYTES,
// which every GPU that loads the library holds until the process exits.
//
// Set-up: the first call on a device (with that device current) looks up the
// array's device address with cudaGetSymbolAddress and remembers it per
// device ordinal.  Make that first call before any stream capture.  In host
// code the array's name is only a host-side stand-in, so the kernels always
// receive the looked-up address.  The remembered address belongs to the
// device's primary context: after cudaDeviceReset (which unloads the library's
// device code) it is stale, so a process that resets a device must not call
// this entry point on that device again.
//
// Sharing: every call on a device uses the same array and finds the previous
// call's contents in it; each call clears the part that must start at zero
// (header and look-back words) on its own stream before launching, the first
// call included, and the rank array is rewritten in full by every call.  Calls
// that overlap on the GPU (different streams, or different host threads on
// the same device) race on the array and must be serialised by the caller.
// Device-side conditions (bad assignment, wait timeout) are recorded in the
// array's header, which the next call clears; this entry point does not
// report them.  After such a condition the outputs are not valid; a caller
// that must detect it uses moe_b200_pack with its own workspace and reads
// moe_b200_workspace_status.
//
// Nothing here calls cudaMalloc, cudaFree or any allocating routine.
#include <mutex>

#include <cuda_runtime.h>

#include "common.cuh"
#include "moe_b200.h"

namespace moe_b200 {
int fail(int code, const char* fmt, ...);
int cuda_fail(cudaError_t err, const char* where);
}  // namespace moe_b200

static __device__ __align__(256) unsigned char g_pack_noalloc_scratch[MOE_B200_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_setup_mutex;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of the built-in scratch on the current device; looked up
// on the first call per device.
int scratch_on_current_device(void** out) {
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return moe_b200::cuda_fail(err, "pack_noalloc: cudaGetDevice");
    if (dev < 0 || dev >= kMaxDevices)
        return moe_b200::fail(MOE_B200_ERR_UNSUPPORTED, "pack_noalloc: device %d beyond %d", dev,
                              kMaxDevices);
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (!g_scratch_addr[dev]) {
        void* p = nullptr;
        err = cudaGetSymbolAddress(&p, g_pack_noalloc_scratch);
        if (err != cudaSuccess) return moe_b200::cuda_fail(err, "pack_noalloc: cudaGetSymbolAddress");
        g_scratch_addr[dev] = p;
    }
    *out = g_scratch_addr[dev];
    return MOE_B200_OK;
}

}  // namespace

extern "C" int moe_b200_pack_noalloc(const void* emb, const int32_t* asgn, const float* wts, int T,
                                     int K, int E, int d, void* packed, float* packed_weights,
                                     int32_t* perm, int32_t* expert_count, int32_t* expert_start,
                                     int32_t* slot_pos, void* stream) {
    using namespace moe_b200;
    if (T < 0 || K < 1 || E < 1 || d < 1)
        return fail(MOE_B200_ERR_INVALID_ARG, "pack_noalloc: need T>=0, K>=1, E>=1, d>=1");
    if (E > MOE_B200_MAX_EXPERTS || K > 32 || int64_t(T) * K > INT32_MAX)
        return fail(MOE_B200_ERR_UNSUPPORTED, "pack_noalloc: shape outside the packing limits");
    const PackPlan plan = plan_pack(T, K, E);
    if (plan.total_bytes > MOE_B200_NOALLOC_SCRATCH_BYTES)
        return fail(MOE_B200_ERR_WORKSPACE,
                    "pack_noalloc: T=%d K=%d E=%d needs %zu bytes of scratch but the built-in scratch "
                    "holds %zu; use moe_b200_pack with a caller-provided workspace",
                    T, K, E, plan.total_bytes, size_t(MOE_B200_NOALLOC_SCRATCH_BYTES));
    void* scratch = nullptr;
    int st = scratch_on_current_device(&scratch);
    if (st != MOE_B200_OK) return st;
    // The header and look-back words must start at zero; the rank array is
    // fully rewritten by every call.
    cudaError_t err = cudaMemsetAsync(scratch, 0, plan.rank_off, static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return cuda_fail(err, "pack_noalloc: clear");
    return moe_b200_pack(emb, asgn, wts, T, K, E, d, packed, packed_weights, perm, expert_count,
                         expert_start, slot_pos, scratch, MOE_B200_NOALLOC_SCRATCH_BYTES, stream);
}
