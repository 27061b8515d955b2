// capi.cu -- extern "C" entry points of libmoe_b200 (declared in
// include/moe_b200.h): argument validation, workspace checks, launches.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <cuda_runtime.h>

#include "common.cuh"
#include "moe_b200.h"

namespace moe_b200 {
cudaError_t launch_pack(const void* emb, const int32_t* asgn, const float* wts, int T, int K,
                        int E, int d, void* packed, float* packed_w, int32_t* perm,
                        int32_t* expert_count, int32_t* expert_start, int32_t* slot_pos,
                        void* ws, cudaStream_t stream);
cudaError_t launch_unpermute(const void* y, const float* packed_w, const int32_t* slot_pos,
                             int T, int K, int d, int dtype, void* out, cudaStream_t stream,
                             const EpWait* wait);

static thread_local char g_last_error[512];

int fail(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
    return code;
}

int cuda_fail(cudaError_t err, const char* where) {
    return fail(MOE_B200_ERR_CUDA, "%s: %s", where, cudaGetErrorString(err));
}

void clear_error() { g_last_error[0] = 0; }
}  // namespace moe_b200

using namespace moe_b200;

extern "C" {

int moe_b200_version(void) { return 100; }

const char* moe_b200_status_string(int status) {
    switch (status) {
        case MOE_B200_OK: return "ok";
        case MOE_B200_ERR_INVALID_ARG: return "invalid argument";
        case MOE_B200_ERR_WORKSPACE: return "workspace missing or too small";
        case MOE_B200_ERR_UNSUPPORTED: return "unsupported shape";
        case MOE_B200_ERR_CUDA: return "CUDA error";
        case MOE_B200_DEV_BAD_ASSIGNMENT: return "device: assignment outside [0, E)";
        case MOE_B200_DEV_WAIT_TIMEOUT: return "device: bounded wait timed out";
        default: return "unknown status";
    }
}

const char* moe_b200_last_error(void) { return g_last_error; }

size_t moe_b200_pack_workspace_bytes(int T, int K, int E) {
    if (T < 0 || K < 1 || E < 1) return 0;
    return plan_pack(T, K, E).total_bytes;
}

int moe_b200_workspace_init(void* workspace, size_t workspace_bytes, void* stream) {
    clear_error();
    if (!workspace || workspace_bytes < sizeof(WsHeader))
        return fail(MOE_B200_ERR_WORKSPACE, "workspace_init: null or smaller than the header");
    cudaError_t err =
        cudaMemsetAsync(workspace, 0, workspace_bytes, static_cast<cudaStream_t>(stream));
    return err == cudaSuccess ? MOE_B200_OK : cuda_fail(err, "workspace_init");
}

int moe_b200_pack(const void* emb, const int32_t* asgn, const float* wts, int T, int K, int E,
                  int d, void* packed, float* packed_weights, int32_t* perm,
                  int32_t* expert_count, int32_t* expert_start, int32_t* slot_pos,
                  void* workspace, size_t workspace_bytes, void* stream) {
    clear_error();
    if (T < 0 || K < 1 || E < 1 || d < 1)
        return fail(MOE_B200_ERR_INVALID_ARG, "pack: need T>=0, K>=1, E>=1, d>=1 (T=%d K=%d E=%d d=%d)",
                    T, K, E, d);
    if (K > 32) return fail(MOE_B200_ERR_UNSUPPORTED, "pack: K=%d exceeds 32", K);
    if (E > MOE_B200_MAX_EXPERTS)
        return fail(MOE_B200_ERR_UNSUPPORTED, "pack: E=%d exceeds %d", E, MOE_B200_MAX_EXPERTS);
    const int64_t TK = int64_t(T) * K;
    if (TK > INT32_MAX) return fail(MOE_B200_ERR_UNSUPPORTED, "pack: T*K=%lld exceeds 2^31-1", (long long)TK);
    if (!expert_count || !expert_start)
        return fail(MOE_B200_ERR_INVALID_ARG, "pack: expert_count / expert_start are required");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (TK == 0) {
        cudaError_t err = cudaMemsetAsync(expert_count, 0, size_t(E) * 4, s);
        if (err == cudaSuccess) err = cudaMemsetAsync(expert_start, 0, size_t(E + 1) * 4, s);
        return err == cudaSuccess ? MOE_B200_OK : cuda_fail(err, "pack (empty)");
    }
    if (!asgn || !perm || (packed && !emb))
        return fail(MOE_B200_ERR_INVALID_ARG, "pack: asgn and perm (and emb when packed is given) are required");
    if (packed_weights && !wts)
        return fail(MOE_B200_ERR_INVALID_ARG, "pack: packed_weights needs wts");
    const size_t need = plan_pack(T, K, E).total_bytes;
    if (!workspace || workspace_bytes < need)
        return fail(MOE_B200_ERR_WORKSPACE, "pack: workspace %zu bytes < required %zu",
                    workspace_bytes, need);
    if (reinterpret_cast<uintptr_t>(workspace) % 256 != 0)
        return fail(MOE_B200_ERR_INVALID_ARG, "pack: workspace must be 256-byte aligned");
    cudaError_t err = launch_pack(emb, asgn, wts, T, K, E, d, packed, packed_weights, perm,
                                  expert_count, expert_start, slot_pos, workspace, s);
    return err == cudaSuccess ? MOE_B200_OK : cuda_fail(err, "pack launch");
}

int moe_b200_workspace_status(void* workspace, size_t workspace_bytes, void* stream,
                              int* device_status) {
    clear_error();
    if (!device_status) return fail(MOE_B200_ERR_INVALID_ARG, "workspace_status: null output");
    if (!workspace || workspace_bytes < sizeof(WsHeader))
        return fail(MOE_B200_ERR_WORKSPACE, "workspace_status: null or smaller than the header");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    uint32_t bits = 0;
    WsHeader* hdr = static_cast<WsHeader*>(workspace);
    cudaError_t err = cudaMemcpyAsync(&bits, &hdr->status, 4, cudaMemcpyDeviceToHost, s);
    if (err == cudaSuccess) err = cudaStreamSynchronize(s);
    if (err == cudaSuccess && bits) err = cudaMemsetAsync(&hdr->status, 0, 4, s);
    if (err == cudaSuccess) err = cudaStreamSynchronize(s);
    if (err != cudaSuccess) return cuda_fail(err, "workspace_status");
    *device_status = int(bits);
    return MOE_B200_OK;
}

int moe_b200_unpermute(const void* y, const float* packed_weights, const int32_t* slot_pos,
                       int T, int K, int d, int dtype, void* out, void* stream) {
    clear_error();
    if (T < 0 || K < 1 || d < 1)
        return fail(MOE_B200_ERR_INVALID_ARG, "unpermute: need T>=0, K>=1, d>=1");
    if (K > 32) return fail(MOE_B200_ERR_UNSUPPORTED, "unpermute: K=%d exceeds 32", K);
    if (dtype != MOE_B200_F16 && dtype != MOE_B200_BF16)
        return fail(MOE_B200_ERR_INVALID_ARG, "unpermute: dtype %d is neither F16 nor BF16", dtype);
    if (int64_t(T) * K > INT32_MAX) return fail(MOE_B200_ERR_UNSUPPORTED, "unpermute: T*K exceeds 2^31-1");
    if (T == 0) return MOE_B200_OK;
    if (!y || !packed_weights || !slot_pos || !out)
        return fail(MOE_B200_ERR_INVALID_ARG, "unpermute: null pointer");
    cudaError_t err = launch_unpermute(y, packed_weights, slot_pos, T, K, d, dtype, out,
                                       static_cast<cudaStream_t>(stream), nullptr);
    return err == cudaSuccess ? MOE_B200_OK : cuda_fail(err, "unpermute launch");
}

}  // extern "C"
