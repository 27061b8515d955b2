// unpermute.cu -- fused weighted unpermute + top-K combine for sm_100a.
//
//   out[t, :] = round16( sum_{k<K} w[p_k] * y[p_k, :] ),  p_k = slot_pos[t*K + k]
//
// Replaces the reference's unpack_combine_kernel (fp32 atomicAdd scatter into
// a zeroed [T, d] fp32 buffer, apps/bench_e2e.cu:136-147) plus its separate
// f32_to_f16_kernel pass (:149-152) and memset (:304).  Here each token
// GATHERS its K rows, so there are no atomics, no fp32 round trip through
// HBM, and the sum is deterministic: fp32, ascending k, one FMA per term.
// HBM traffic is the algorithmic minimum: T*K*d*2 bytes read + T*d*2 written.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdlib>

#include <cuda_runtime.h>

#include "common.cuh"

namespace moe_b200 {

template <int DT>
__device__ __forceinline__ void acc_vec(float (&a)[8], float w, const uint4& v) {
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int h = 0; h < 4; ++h) {
        float2 f;
        if (DT == MOE_B200_F16) {
            __half2 x = *reinterpret_cast<const __half2*>(&u[h]);
            f = __half22float2(x);
        } else {
            __nv_bfloat162 x = *reinterpret_cast<const __nv_bfloat162*>(&u[h]);
            f = __bfloat1622float2(x);
        }
        a[2 * h] = __fmaf_rn(w, f.x, a[2 * h]);
        a[2 * h + 1] = __fmaf_rn(w, f.y, a[2 * h + 1]);
    }
}

template <int DT>
__device__ __forceinline__ uint4 pack_vec(const float (&a)[8]) {
    uint32_t u[4];
#pragma unroll
    for (int h = 0; h < 4; ++h) {
        if (DT == MOE_B200_F16) {
            __half2 x = __floats2half2_rn(a[2 * h], a[2 * h + 1]);
            u[h] = *reinterpret_cast<uint32_t*>(&x);
        } else {
            __nv_bfloat162 x = __floats2bfloat162_rn(a[2 * h], a[2 * h + 1]);
            u[h] = *reinterpret_cast<uint32_t*>(&x);
        }
    }
    return make_uint4(u[0], u[1], u[2], u[3]);
}

// One warp per token.  VPL 16-byte vectors per lane per pass; the K source
// rows are fetched KB at a time so that KB*VPL loads are in flight per lane.
template <int DT, int VPL, int KB>
__global__ void __launch_bounds__(256)
unpermute_kernel(const uint4* __restrict__ y, const float* __restrict__ packed_w,
                 const int32_t* __restrict__ slot_pos, int T, int K, int nvec,
                 uint4* __restrict__ out) {
    pdl_wait_primary();
    const int lane = threadIdx.x & 31;
    const int warps_per_cta = blockDim.x >> 5;
    const int64_t gw = int64_t(blockIdx.x) * warps_per_cta + (threadIdx.x >> 5);
    const int64_t nw = int64_t(gridDim.x) * warps_per_cta;

    for (int64_t t = gw; t < T; t += nw) {
        int32_t p_lane = lane < K ? __ldg(slot_pos + t * K + lane) : -1;
        float w_lane = p_lane >= 0 ? __ldg(packed_w + p_lane) : 0.f;
        for (int c0 = 0; c0 < nvec; c0 += 32 * VPL) {
            float acc[VPL][8];
#pragma unroll
            for (int j = 0; j < VPL; ++j)
#pragma unroll
                for (int h = 0; h < 8; ++h) acc[j][h] = 0.f;

            for (int kb = 0; kb < K; kb += KB) {
                uint4 v[KB][VPL];
                int32_t p[KB];
#pragma unroll
                for (int q = 0; q < KB; ++q) {
                    p[q] = __shfl_sync(0xffffffffu, p_lane, (kb + q) & 31);
                    if (kb + q >= K) p[q] = -1;
#pragma unroll
                    for (int j = 0; j < VPL; ++j) {
                        int i = c0 + j * 32 + lane;
                        if (p[q] >= 0 && i < nvec) v[q][j] = ld_nc_v4(y + int64_t(p[q]) * nvec + i);
                    }
                }
#pragma unroll
                for (int q = 0; q < KB; ++q) {
                    float w = __shfl_sync(0xffffffffu, w_lane, (kb + q) & 31);
                    if (p[q] < 0) continue;
#pragma unroll
                    for (int j = 0; j < VPL; ++j) acc_vec<DT>(acc[j], w, v[q][j]);
                }
            }
            uint4* dst = out + t * nvec;
#pragma unroll
            for (int j = 0; j < VPL; ++j) {
                int i = c0 + j * 32 + lane;
                if (i < nvec) st_v4(dst + i, pack_vec<DT>(acc[j]));
            }
        }
    }
}

// TMA bulk-copy pipeline: per CTA one producer warp and kConsumerWarps
// consumer warps.  For each of the CTA's tokens the producer's lanes k < K
// issue one cp.async.bulk of row y[p_k] (d*2 bytes) into a shared-memory
// stage; the consumers wait on the stage's mbarrier, accumulate the K rows in
// fp32 (ascending k, one FMA per term), round once and store the output row.
// `stages` stages per CTA keep stages*K rows in flight with no register cost.
constexpr int kConsumerWarps = 8;
constexpr int kBulkThreads = (kConsumerWarps + 1) * 32;

// Expert parallel: the rows of y arrive from the peers; lanes of one warp
// wait (bounded) until every rank's back flag reached the epoch, then order
// the acquire before this thread's later bulk-copy reads of y.
__device__ __forceinline__ void wait_back_flags(const EpWait& wt, int lane, uint32_t* dev_status) {
    for (int i = lane; i < wt.n; i += 32) {
        const uint64_t t0 = globaltimer_ns();
        while (ld_acquire_sys(wt.flags + i) < wt.epoch) {
            if (globaltimer_ns() - t0 > wt.timeout_ns) {
                atomicOr(dev_status, MOE_B200_DEV_WAIT_TIMEOUT);
                break;
            }
            __nanosleep(64);
        }
    }
    __syncwarp();
    fence_proxy_async_global();
}

// Stand-alone form of the same wait, for the unpermute kernels that are not
// bulk-copy pipelines.
__global__ void ep_wait_back_kernel(EpWait wt, uint32_t* __restrict__ dev_status) {
    pdl_wait_primary();
    if (threadIdx.x < 32) wait_back_flags(wt, threadIdx.x, dev_status);
    __threadfence_system();
}

template <int DT>
__global__ void __launch_bounds__(kBulkThreads)
unpermute_bulk_kernel(const uint16_t* __restrict__ y, const float* __restrict__ packed_w,
                      const int32_t* __restrict__ slot_pos, int T, int K, int d, int stages,
                      uint4* __restrict__ out, uint32_t* __restrict__ dev_status, EpWait wt) {
    extern __shared__ __align__(128) unsigned char smem[];
    const uint32_t rowb = uint32_t(d) * 2;
    const size_t stage_bytes = size_t(K) * rowb;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + size_t(stages) * stage_bytes);
    uint64_t* empty = full + stages;
    float* sw = reinterpret_cast<float*>(empty + stages);  // [stages][K] weights
    int32_t* sp = reinterpret_cast<int32_t*>(sw + stages * K);  // [stages][K] rows

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    pdl_wait_primary();
    if (tid == 0) {
        for (int s = 0; s < stages; ++s) {
            mbar_init(full + s, 1);
            mbar_init(empty + s, kConsumerWarps);
        }
        mbar_fence_init();
    }
    __syncthreads();

    if (warp == kConsumerWarps) {
        // Producer.  The CTA's tokens are t_i = blockIdx.x + i * gridDim.x.
        // Lane l covers slot k = l % K of token i = g * G + l / K of group g
        // (G = 32 / K tokens per group), so one load round trip fetches the
        // row indices and weights of G tokens; the next group's are in flight
        // while this group's copies are issued.
        const int G = 32 / K;
        const int gk = lane % K, gi = lane / K;
        const bool lane_used = gi < G;
        const int64_t n_mine = (T - 1 - int64_t(blockIdx.x)) / gridDim.x + 1;  // tokens of this CTA
        if (wt.flags) wait_back_flags(wt, lane, dev_status);
        auto fetch_p = [&](int64_t g) -> int32_t {
            const int64_t i = g * G + gi;
            if (!lane_used || i >= n_mine) return -1;
            const int64_t t = int64_t(blockIdx.x) + i * gridDim.x;
            return __ldg(slot_pos + t * K + gk);
        };
        auto fetch_w = [&](int32_t p) -> float { return p >= 0 ? __ldg(packed_w + p) : 0.f; };
        // indices run two groups ahead, weights one group ahead, so no
        // dependent load sits on the per-group path
        int32_t p_cur = fetch_p(0);
        int32_t p_nxt = fetch_p(1);
        float w_cur = fetch_w(p_cur);
        float w_nxt;
        bool ok = true;
        uint32_t issued = 0;  // stages filled
        for (int64_t g = 0; ok && g * G < n_mine; ++g) {
            const int32_t p_nn = fetch_p(g + 2);
            w_nxt = fetch_w(p_nxt);
            for (int q = 0; q < G; ++q) {
                const int64_t i = g * G + q;
                if (i >= n_mine) break;
                const int s = int(i % stages);
                const uint32_t ph = uint32_t(i / stages) & 1u;
                if (!mbar_wait(empty + s, ph ^ 1u)) {
                    if (lane == 0) atomicOr(dev_status, MOE_B200_DEV_WAIT_TIMEOUT);
                    ok = false;
                    break;
                }
                const bool mine = lane_used && gi == q;
                if (mine) {
                    sw[s * K + gk] = w_cur;
                    sp[s * K + gk] = p_cur;
                }
                const uint32_t valid = __ballot_sync(0xffffffffu, mine && p_cur >= 0);
                __syncwarp();
                if (lane == 0) mbar_arrive_expect_tx(full + s, uint32_t(__popc(valid)) * rowb);
                __syncwarp();
                if (mine && p_cur >= 0)
                    bulk_g2s(smem + size_t(s) * stage_bytes + size_t(gk) * rowb,
                             y + int64_t(p_cur) * d, rowb, full + s);
                issued = uint32_t(i + 1);
            }
            p_cur = p_nxt;
            w_cur = w_nxt;
            p_nxt = p_nn;
        }
        // after an abort, no row copy may still be landing in shared memory
        // when the CTA exits (normally the consumers waited for every one)
        if (!ok && lane == 0) drain_stages(full, issued, stages);
    } else {
        const int ctid = tid;  // 0 .. 32*kConsumerWarps-1
        const int nvec = d >> 3;
        int64_t t = blockIdx.x;
        for (int i = 0; t < T; t += gridDim.x, ++i) {
            const int s = i % stages;
            const uint32_t ph = uint32_t(i / stages) & 1u;
            if (!mbar_wait(full + s, ph)) {
                if (ctid == 0) atomicOr(dev_status, MOE_B200_DEV_WAIT_TIMEOUT);
                break;
            }
            const unsigned char* st = smem + size_t(s) * stage_bytes;
            uint4* dst = out + t * nvec;
            for (int v = ctid; v < nvec; v += 32 * kConsumerWarps) {
                float acc[8];
#pragma unroll
                for (int h = 0; h < 8; ++h) acc[h] = 0.f;
                for (int k = 0; k < K; ++k) {
                    if (sp[s * K + k] < 0) continue;
                    const uint4 x = *reinterpret_cast<const uint4*>(st + size_t(k) * rowb + size_t(v) * 16);
                    acc_vec<DT>(acc, sw[s * K + k], x);
                }
                st_v4(dst + v, pack_vec<DT>(acc));
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(empty + s);
        }
    }
}

// Fallback for rows that are not 16-byte multiples / not 16-byte aligned.
template <int DT>
__global__ void __launch_bounds__(256)
unpermute_scalar_kernel(const uint16_t* __restrict__ y, const float* __restrict__ packed_w,
                        const int32_t* __restrict__ slot_pos, int T, int K, int d,
                        uint16_t* __restrict__ out) {
    pdl_wait_primary();
    const int64_t n = int64_t(T) * d;
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += int64_t(gridDim.x) * blockDim.x) {
        int64_t t = i / d, c = i % d;
        float a = 0.f;
        for (int k = 0; k < K; ++k) {
            int32_t p = slot_pos[t * K + k];
            if (p < 0) continue;
            uint16_t raw = y[int64_t(p) * d + c];
            float f;
            if (DT == MOE_B200_F16) f = __half2float(*reinterpret_cast<const __half*>(&raw));
            else f = __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(&raw));
            a = __fmaf_rn(packed_w[p], f, a);
        }
        if (DT == MOE_B200_F16) {
            __half h = __float2half_rn(a);
            out[i] = *reinterpret_cast<uint16_t*>(&h);
        } else {
            __nv_bfloat16 h = __float2bfloat16_rn(a);
            out[i] = *reinterpret_cast<uint16_t*>(&h);
        }
    }
}

static int sm_count_unperm() {
    int dev = 0, n = 148;
    if (cudaGetDevice(&dev) == cudaSuccess)
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n > 0 ? n : 148;
}

static int bulk_smem_bytes(int K, int d, int stages) {
    return stages * (K * d * 2 + 2 * 8 + K * 8) + 128;
}

cudaError_t launch_unpermute(const void* y, const float* packed_w, const int32_t* slot_pos,
                             int T, int K, int d, int dtype, void* out, cudaStream_t stream,
                             const EpWait* wait) {
    EpWait wt{};
    if (wait) wt = *wait;
    const bool vec = (d % 8 == 0) && (reinterpret_cast<uintptr_t>(y) % 16 == 0) &&
                     (reinterpret_cast<uintptr_t>(out) % 16 == 0);
    const int threads = 256;
    const int sms = sm_count_unperm();
    // Bulk-copy pipeline when at least 2 stages of K rows fit in shared memory.
    const size_t stage = size_t(K) * d * 2;
    int stages = stage > 0 ? int((200 * 1024) / stage) : 0;
    if (stages > 4) stages = 4;
    const char* sel = getenv("MOE_B200_UNPERMUTE");
    const bool want_bulk = !(sel && sel[0] == 'r');
    if (vec && want_bulk && stages >= 2) {
        uint32_t* st = device_status_word();
        if (!st) return cudaErrorInvalidDevice;
        const int smem = bulk_smem_bytes(K, d, stages);
        auto kern = dtype == MOE_B200_F16 ? unpermute_bulk_kernel<MOE_B200_F16>
                                          : unpermute_bulk_kernel<MOE_B200_BF16>;
        cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (err != cudaSuccess) return err;
        int per_sm = 0;
        err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kBulkThreads, smem);
        if (err != cudaSuccess) return err;
        if (per_sm < 1) per_sm = 1;
        int64_t grid = int64_t(sms) * per_sm;
        if (grid > T) grid = T;
        cudaLaunchConfig_t cfg = pdl_config(dim3(unsigned(grid)), dim3(kBulkThreads), smem, stream);
        cudaLaunchAttribute attr = pdl_attr();
        cfg.attrs = &attr;
        cfg.numAttrs = 1;
        return cudaLaunchKernelEx(&cfg, kern, static_cast<const uint16_t*>(y), packed_w, slot_pos, T, K,
                                  d, stages, static_cast<uint4*>(out), st, wt);
    }
    if (wt.flags) {
        uint32_t* st = device_status_word();
        if (!st) return cudaErrorInvalidDevice;
        cudaLaunchConfig_t cfg = pdl_config(dim3(1), dim3(32), 0, stream);
        cudaLaunchAttribute attr = pdl_attr();
        cfg.attrs = &attr;
        cfg.numAttrs = 1;
        cudaError_t err = cudaLaunchKernelEx(&cfg, ep_wait_back_kernel, wt, st);
        if (err != cudaSuccess) return err;
    }
    if (vec) {
        const int warps_per_cta = threads / 32;
        int64_t want = (int64_t(T) + warps_per_cta - 1) / warps_per_cta;
        int64_t cap = int64_t(sms) * 64;
        int grid = int(want < cap ? want : cap);
        if (grid < 1) grid = 1;
        cudaLaunchConfig_t cfg = pdl_config(dim3(grid), dim3(threads), 0, stream);
        cudaLaunchAttribute attr = pdl_attr();
        cfg.attrs = &attr;
        cfg.numAttrs = 1;
        auto kern = dtype == MOE_B200_F16 ? unpermute_kernel<MOE_B200_F16, 2, 4>
                                          : unpermute_kernel<MOE_B200_BF16, 2, 4>;
        return cudaLaunchKernelEx(&cfg, kern, static_cast<const uint4*>(y), packed_w, slot_pos, T, K,
                                  d / 8, static_cast<uint4*>(out));
    } else {
        int64_t n = int64_t(T) * d;
        int64_t want = (n + threads - 1) / threads;
        int64_t cap = int64_t(sms) * 32;
        int grid = int(want < cap ? want : cap);
        if (grid < 1) grid = 1;
        cudaLaunchConfig_t cfg = pdl_config(dim3(grid), dim3(threads), 0, stream);
        cudaLaunchAttribute attr = pdl_attr();
        cfg.attrs = &attr;
        cfg.numAttrs = 1;
        auto kern = dtype == MOE_B200_F16 ? unpermute_scalar_kernel<MOE_B200_F16>
                                          : unpermute_scalar_kernel<MOE_B200_BF16>;
        return cudaLaunchKernelEx(&cfg, kern, static_cast<const uint16_t*>(y), packed_w, slot_pos, T, K,
                                  d, static_cast<uint16_t*>(out));
    }
    return cudaGetLastError();
}

}  // namespace moe_b200
