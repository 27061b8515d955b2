// ep_layout.cu -- expert-parallel exchange layout, computed on the device.
//
// Given every rank's per-expert row counts (all_counts[g][e], gathered with
// one collective), rank `rank` needs
//   send_counts[g]  rows of its packed buffer that go to rank g: the rows of
//                   g's contiguous expert range (the packed buffer is already
//                   the rank-major send buffer, so no repack);
//   recv_counts[g]  rows it receives from rank g;
//   seg_start / seg_expert  the segments of its receive buffer, which is
//                   sender-major then expert-major (as in the reference,
//                   apps/bench_prefill.cu:642-682): segment g*L + j holds the
//                   rows sender g routed to local expert j (L = local experts),
//                   ready for moe_b200_grouped_swiglu.
// The reference computes the split sizes on the host after a D2H copy
// (apps/bench_prefill.cu:768-788) and builds the FFN problem list on the
// host every round (:812-852).
#include <cuda_runtime.h>

#include "common.cuh"

namespace moe_b200 {

constexpr int kMaxRanks = 64;
struct RankBounds {
    int first[kMaxRanks + 1];
};

__global__ void __launch_bounds__(256)
ep_layout_kernel(const int32_t* __restrict__ all_counts, int N, int E, int rank, RankBounds b,
                 int32_t* __restrict__ seg_start, int32_t* __restrict__ seg_expert,
                 int32_t* __restrict__ send_counts, int32_t* __restrict__ recv_counts) {
    pdl_wait_primary();
    const int tid = threadIdx.x;
    const int lo = b.first[rank], hi = b.first[rank + 1], L = hi - lo;
    // send / recv counts: one thread per peer
    for (int g = tid; g < N; g += blockDim.x) {
        int s = 0, r = 0;
        for (int e = b.first[g]; e < b.first[g + 1]; ++e) s += all_counts[rank * E + e];
        for (int e = lo; e < hi; ++e) r += all_counts[g * E + e];
        send_counts[g] = s;
        recv_counts[g] = r;
    }
    // segment offsets: exclusive scan over (g, j) in row-major order
    const int nseg = N * L;
    __shared__ int32_t warp_tot[8];
    __shared__ int32_t carry;
    if (tid == 0) carry = 0;
    __syncthreads();
    const int lane = tid & 31, warp = tid >> 5;
    for (int base = 0; base < nseg; base += blockDim.x) {
        const int i = base + tid;
        int32_t v = 0;
        if (i < nseg) {
            const int g = i / L, j = i % L;
            v = all_counts[g * E + lo + j];
            seg_expert[i] = j;
        }
        int32_t incl = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            int32_t n = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += n;
        }
        if (lane == 31) warp_tot[warp] = incl;
        __syncthreads();
        int32_t off = carry;
        for (int w = 0; w < warp; ++w) off += warp_tot[w];
        if (i < nseg) seg_start[i] = off + incl - v;
        __syncthreads();
        if (tid == blockDim.x - 1) carry = off + incl;
        __syncthreads();
    }
    if (tid == 0) seg_start[nseg] = carry;
}

int fail(int code, const char* fmt, ...);
int cuda_fail(cudaError_t err, const char* where);

}  // namespace moe_b200

extern "C" int moe_b200_ep_layout(const int32_t* all_counts, int nranks, int E, int rank,
                                  const int32_t* expert_first, int32_t* seg_start,
                                  int32_t* seg_expert, int32_t* send_counts, int32_t* recv_counts,
                                  void* stream) {
    using namespace moe_b200;
    if (nranks < 1 || nranks > kMaxRanks || E < 1 || rank < 0 || rank >= nranks)
        return fail(MOE_B200_ERR_INVALID_ARG, "ep_layout: need 1 <= nranks <= %d, 0 <= rank < nranks, E >= 1",
                    kMaxRanks);
    if (!all_counts || !expert_first || !seg_start || !seg_expert || !send_counts || !recv_counts)
        return fail(MOE_B200_ERR_INVALID_ARG, "ep_layout: null pointer");
    RankBounds b{};
    if (expert_first[0] != 0 || expert_first[nranks] != E)
        return fail(MOE_B200_ERR_INVALID_ARG, "ep_layout: expert_first must run from 0 to E");
    for (int g = 0; g <= nranks; ++g) {
        b.first[g] = expert_first[g];
        if (g > 0 && expert_first[g] < expert_first[g - 1])
            return fail(MOE_B200_ERR_INVALID_ARG, "ep_layout: expert_first must be non-decreasing");
    }
    cudaLaunchConfig_t cfg = pdl_config(dim3(1), dim3(256), 0, static_cast<cudaStream_t>(stream));
    cudaLaunchAttribute attr = pdl_attr();
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    cudaError_t err = cudaLaunchKernelEx(&cfg, ep_layout_kernel, all_counts, nranks, E, rank, b, seg_start,
                                         seg_expert, send_counts, recv_counts);
    return err == cudaSuccess ? MOE_B200_OK : cuda_fail(err, "ep_layout launch");
}
