// router.cu -- MoE router on the tcgen05 tensor cores (sm_100a): gate GEMM,
// softmax over all experts and top-K in one kernel, logits never leave the
// SM (they live in TMEM between the MMAs and the epilogue).
//
// Reference semantics (apps/bench_e2e.cu:95-130, fused_route_kernel; the
// unfused chain gate_kernel / softmax_kernel / topk_kernel :51-93 computes the
// same): logit[t, e] = sum_i fp32(emb[t, i]) * W_gate[i*E + e]; softmax with
// the maximum subtracted, expf, a sum in ascending e and one division per
// expert; then K rounds of "argmax, ties to the lowest index, remove".
//
// B200 design.  The gate GEMM is [T, d] x [d, E] with E <= 256: a GEMM with
// a narrow N, so each CTA owns 128 tokens (TMEM lanes) and the whole expert
// range (N = E rounded up to 16 columns).  The fp32 gate weights are
// prepared once into 16-bit pieces of the embeddings' own type,
//     W * 2^s  =  W1 + W2 (+ W3)
// (fp16: two pieces after a power-of-two pre-scale that puts max|W| just
// under 2^14 so the second piece stays normal; bf16: three pieces, bf16 has
// the fp32 exponent range), transposed to K-major [piece][E_pad][d].  The MMA
// (kind::f16, fp32 accumulate) then takes the embeddings straight from HBM
// through TMA, unconverted; every product of a 16-bit embedding and a 16-bit
// piece is exact in fp32, so the accumulated logits carry fp32-level error
// (the residual of the split is below 2^-22 of max|W|).  The epilogue warps
// (one token per thread) read the logits back from TMEM three times: maximum,
// sum of exponentials, then probabilities fed into a K-entry insertion list.
//
// Roles per CTA (192 threads): warp 0 TMA producer (A 128 x 64 + P pieces of
// E_pad x 64 per stage, 128-byte swizzle), warp 1 TMEM allocator and
// single-thread MMA issuer, warps 2-5 epilogue.  All waits are bounded.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "common.cuh"
#include "tcgen05.cuh"

namespace moe_b200 {

int fail(int code, const char* fmt, ...);
int cuda_fail(cudaError_t err, const char* where);

namespace {

constexpr int kRtThreads = 320;  // warp 0 TMA, warp 1 MMA, warps 2-9 epilogue
constexpr int kRtTileM = 128;
constexpr int kRtTileK = 64;
constexpr uint32_t kRtABytes = kRtTileM * kRtTileK * 2;  // 16 KB
constexpr int kRtMaxStages = 4;
constexpr size_t kRtStageBudget = 200 * 1024;
constexpr uint32_t kRouterMagic = 0x5254524Du;  // "MRTR"
constexpr size_t kRouterHeaderBytes = 256;

// Header of a prepared weight buffer; the pieces follow at kRouterHeaderBytes.
struct RouterHeader {
    uint32_t magic;
    int32_t d, E, E_pad, pieces, dtype;
    int32_t scale_exp;     // pieces sum to W * 2^scale_exp
    uint32_t absmax_bits;  // max |W| as float bits (scratch of the prepare step)
};

struct RouteSmem {
    float merge_v[256][8];  // each epilogue thread's top-K over its expert range
    int merge_i[256][8];
    float merge_f[256];     // each epilogue thread's partial sum of exponentials
    float row_max[128];
    uint64_t full[kRtMaxStages];
    uint64_t empty[kRtMaxStages];
    uint64_t done;
    uint32_t tmem_base;
    int abort_flag;
};

inline int round_up16(int x) { return (x + 15) & ~15; }
inline int pieces_for(int dtype) { return dtype == MOE_B200_BF16 ? 3 : 2; }
__host__ __device__ inline uint32_t stage_bytes(int E_pad, int P) { return kRtABytes + uint32_t(P) * E_pad * kRtTileK * 2; }

// ------------------------------------------------------------- prepare ----

__global__ void router_absmax_kernel(const float* __restrict__ w, int64_t n, RouterHeader* hdr) {
    float m = 0.f;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
        m = fmaxf(m, fabsf(w[i]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    // non-negative floats order like their bit patterns
    if ((threadIdx.x & 31) == 0) atomicMax(&hdr->absmax_bits, __float_as_uint(m));
}

template <int DT>
__device__ __forceinline__ uint16_t to16(float v) {
    if (DT == MOE_B200_BF16) {
        __nv_bfloat16 b = __float2bfloat16_rn(v);
        return *reinterpret_cast<uint16_t*>(&b);
    } else {
        __half h = __float2half_rn(v);
        return *reinterpret_cast<uint16_t*>(&h);
    }
}
template <int DT>
__device__ __forceinline__ float from16(uint16_t v) {
    if (DT == MOE_B200_BF16) return __bfloat162float(*reinterpret_cast<__nv_bfloat16*>(&v));
    return __half2float(*reinterpret_cast<__half*>(&v));
}

// 32 x 32 transposing split: w [d, E] (row i = input feature) -> pieces
// [P][E_pad][d], rows e >= E zero.  Block (32, 8).
template <int DT>
__global__ void router_split_kernel(const float* __restrict__ w, int d, int E, int E_pad, RouterHeader* hdr,
                                    uint16_t* __restrict__ out) {
    __shared__ float tile[32][33];
    const int i0 = blockIdx.x * 32, e0 = blockIdx.y * 32;
    for (int r = threadIdx.y; r < 32; r += 8) {
        const int i = i0 + r, e = e0 + threadIdx.x;
        tile[r][threadIdx.x] = (i < d && e < E) ? w[int64_t(i) * E + e] : 0.f;
    }
    __syncthreads();
    int s = 0;
    if (DT == MOE_B200_F16) {
        const float m = __uint_as_float(hdr->absmax_bits);
        if (m > 0.f) {
            int ex;
            frexpf(m, &ex);  // m < 2^ex
            s = 14 - ex;
            s = s > 100 ? 100 : (s < -100 ? -100 : s);
        }
    }
    if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0 && threadIdx.y == 0) {
        hdr->scale_exp = s;
        hdr->magic = kRouterMagic;
    }
    const int P = DT == MOE_B200_BF16 ? 3 : 2;
    const int64_t piece_elems = int64_t(E_pad) * d;
    for (int r = threadIdx.y; r < 32; r += 8) {
        const int e = e0 + r, i = i0 + threadIdx.x;
        if (e >= E_pad || i >= d) continue;
        float rem = ldexpf(tile[threadIdx.x][r], s);
        for (int p = 0; p < P; ++p) {
            const uint16_t q = to16<DT>(rem);
            out[p * piece_elems + int64_t(e) * d + i] = q;
            rem -= from16<DT>(q);  // exact: the piece holds rem's leading bits
        }
    }
}

// --------------------------------------------------------------- route ----

__device__ __forceinline__ uint32_t rt_cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t rt_cluster_id() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void rt_cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t rt_mapa(uint32_t smem_addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
    return r;
}

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Inserts (v, i) into a descending list of K entries, after every entry
// that is not smaller (callers insert in ascending i, so equal values keep
// ascending i).  Below the insertion point every entry moves down one; the
// last falls off.
template <int K>
__device__ __forceinline__ void topk_insert(float (&bv)[K], int (&bi)[K], float v, int i) {
    bool shift = false;
#pragma unroll
    for (int k = 0; k < K; ++k) {
        const bool take = shift || v > bv[k];
        const float tv = bv[k];
        const int ti = bi[k];
        bv[k] = take ? v : tv;
        bi[k] = take ? i : ti;
        v = take ? tv : v;
        i = take ? ti : i;
        shift = take;
    }
}

// One CTA per (128-token tile, K slice).  With nsplit > 1 the CTAs of a
// tile form a cluster: each accumulates the logits of its slice of the d
// input features in its own TMEM, and CTA c finishes token rows
// [c*R, c*R + R), R = 128 / nsplit: every CTA stores the partial logits of
// each row into the (by then idle) stage buffers of the CTA that finishes
// it, over distributed shared memory, and that CTA's epilogue threads add
// the slices in rank order.
template <int DT, int K>
__global__ void __launch_bounds__(kRtThreads, 1)
route_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
             const RouterHeader* __restrict__ hdr, int T, int d, int E, int E_pad, int P, int stages,
             int nsplit, uint32_t area_bytes, int32_t* __restrict__ assignments, float* __restrict__ weights,
             uint32_t* __restrict__ dev_status) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* base = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbytes = stage_bytes(E_pad, P);
    const uint32_t piece_bytes = uint32_t(E_pad) * kRtTileK * 2;
    // stage buffers, then (over the same bytes, once the main loop is over)
    // the logit rows of the R rows this CTA finishes, one per row and K
    // slice, stride E_pad + 4 floats for conflict-free 16-byte accesses
    RouteSmem* ctl = reinterpret_cast<RouteSmem*>(base + area_bytes);
    float* s_logit = reinterpret_cast<float*>(base);
    const int lstride = E_pad + 4;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    volatile int* abort_flag = &ctl->abort_flag;
    const uint32_t crank = nsplit > 1 ? rt_cluster_rank() : 0u;
    const int tile = nsplit > 1 ? int(rt_cluster_id()) : int(blockIdx.x);
    const int row0 = tile * kRtTileM;
    const int nk = (d + kRtTileK - 1) / kRtTileK;
    const int kb0 = int(crank) * nk / nsplit, kb1 = (int(crank) + 1) * nk / nsplit;
    // The P pieces' B tiles are contiguous in shared memory (8-row swizzle
    // atoms), so one MMA with N = P * E_pad (two when that exceeds 256)
    // multiplies the A slice by every piece at once: A is read from shared
    // memory once per K step instead of P times.  Accumulator column
    // p * E_pad + e holds piece p's share of logit e.
    const int ntot = P * E_pad;
    const int n0 = ntot <= 256 ? ntot : ((ntot / 2 + 15) & ~15);  // first MMA's N
    uint32_t ncols = 32;
    while (ncols < uint32_t(ntot)) ncols <<= 1;

    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; ++s) {
            mbar_init(&ctl->full[s], 1);
            mbar_init(&ctl->empty[s], 1);
        }
        mbar_init(&ctl->done, 1);
        ctl->abort_flag = 0;
        mbar_fence_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tmap_x);
        prefetch_tmap(&tmap_w);
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(&ctl->tmem_base)),
                     "r"(ncols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = ctl->tmem_base;

    // The prepared weights must match this call's shape and type.
    const bool hdr_ok = hdr->magic == kRouterMagic && hdr->d == d && hdr->E == E && hdr->E_pad == E_pad &&
                        hdr->pieces == P && hdr->dtype == DT;
    if (!hdr_ok) {
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicOr(dev_status, MOE_B200_DEV_BAD_WEIGHTS);
    } else if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            uint32_t issued = 0;
            for (int kb = kb0; kb < kb1; ++kb) {
                const int j = kb - kb0, st = j % stages;
                if (!wait_or_abort(&ctl->empty[st], ((j / stages) & 1) ^ 1, abort_flag, dev_status)) break;
                unsigned char* sa = base + st * sbytes;
                mbar_arrive_expect_tx(&ctl->full[st], sbytes);
                tma_load_2d(sa, &tmap_x, kb * kRtTileK, row0, &ctl->full[st]);
                for (int p = 0; p < P; ++p)
                    tma_load_2d(sa + kRtABytes + p * piece_bytes, &tmap_w, kb * kRtTileK, p * E_pad,
                                &ctl->full[st]);
                issued = uint32_t(j + 1);
            }
            if (*abort_flag) drain_stages(ctl->full, issued, stages);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            const int fmt = DT == MOE_B200_BF16 ? 1 : 0;
            const uint32_t idesc0 = umma_idesc_mn(fmt, kRtTileM, n0);
            const uint32_t idesc1 = umma_idesc_mn(fmt, kRtTileM, ntot - n0);
            bool ok = true;
            for (int kb = kb0; kb < kb1; ++kb) {
                const int j = kb - kb0, st = j % stages;
                if (!wait_or_abort(&ctl->full[st], (j / stages) & 1, abort_flag, dev_status)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t a_addr = smem_u32(base + st * sbytes);
#pragma unroll
                for (int kk = 0; kk < kRtTileK / 16; ++kk) {
                    const uint64_t ad = umma_desc_sw128(a_addr + kk * 32);
                    const uint32_t b_addr = a_addr + kRtABytes + kk * 32;
                    const uint32_t accum = (j > 0 || kk > 0) ? 1u : 0u;
                    umma_f16(tmem, ad, umma_desc_sw128(b_addr), idesc0, accum);
                    if (n0 < ntot)  // rows n0.. of the stacked B tile: n0 / 8 swizzle atoms further
                        umma_f16(tmem + uint32_t(n0), ad, umma_desc_sw128(b_addr + uint32_t(n0) * 128u), idesc1,
                                 accum);
                }
                umma_commit(&ctl->empty[st]);
            }
            if (ok) umma_commit(&ctl->done);  // also when this slice is empty
        }
    }
    // ---------------- epilogue ----------------
    // Logit rows live over the (then idle) stage buffers: slot q holds the
    // partial logits of K slice q, finished-row j at slot q + j * lstride
    // floats.
    const bool epi = warp >= 2;
    const bool copier = warp >= 2 && warp < 6;  // one warp per TMEM lane quadrant
    const int quad = warp & 3;
    const int R = kRtTileM / nsplit;  // rows this CTA finishes
    const int slot_floats = R * lstride;
    bool have = false;
    if (copier && hdr_ok && wait_or_abort(&ctl->done, 0, abort_flag, dev_status)) {
        tc_fence_after();
        have = true;
    }
    // A peer may write into this CTA's stage buffers only once its main
    // loop is over: every CTA passes this barrier after its own
    // accumulation completed.
    if (nsplit > 1) rt_cluster_sync();
    if (have) {
        // this CTA's partial logits of row r (= TMEM lane) -> slot crank of
        // the CTA finishing r (peers over distributed shared memory, the
        // own rows locally)
        const int r = quad * 32 + lane;
        const uint32_t dst_cta = uint32_t(r / R);
        const uint32_t t_row = tmem + (uint32_t(quad * 32) << 16);
        float* dst_row = s_logit + int(crank) * slot_floats + (r % R) * lstride;
        const uint32_t dst_cl = dst_cta != crank ? rt_mapa(smem_u32(dst_row), dst_cta) : 0u;
        for (int c = 0; c < E_pad; c += 16) {
            // every piece's columns in flight at once, one wait
            uint32_t v[16], w[2][16];
            tmem_ld16(t_row + c, v);
#pragma unroll
            for (int p = 1; p < 3; ++p)
                if (p < P) tmem_ld16(t_row + uint32_t(p * E_pad) + c, w[p - 1]);
            tmem_wait_ld();
#pragma unroll
            for (int p = 1; p < 3; ++p) {  // hi + mid + lo pieces, in order
                if (p >= P) break;
#pragma unroll
                for (int q = 0; q < 16; ++q)
                    v[q] = __float_as_uint(__uint_as_float(v[q]) + __uint_as_float(w[p - 1][q]));
            }
#pragma unroll
            for (int q = 0; q < 16; q += 4) {
                if (dst_cta == crank) {
                    *reinterpret_cast<uint4*>(dst_row + c + q) = make_uint4(v[q], v[q + 1], v[q + 2], v[q + 3]);
                } else {
                    asm volatile("st.shared::cluster.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(dst_cl + uint32_t(c + q) * 4u),
                                 "r"(v[q]), "r"(v[q + 1]), "r"(v[q + 2]), "r"(v[q + 3])
                                 : "memory");
                }
            }
        }
    }
    if (nsplit > 1) rt_cluster_sync();  // every slice of this CTA's rows is in its slots
    // Softmax / top-K of the R rows: TPR = 256 / R threads per row (2, 4 or
    // 8), each over a contiguous range of experts (a multiple of 4 but the
    // last), merged through shared memory in ascending range order --
    // several threads per row hide the latency of the serial insertion
    // chains.
    if (epi) {
        const int et = threadIdx.x - 64;   // 0..255
        const int j = et % R;              // finished row; consecutive lanes, consecutive rows
        const int part = et / R;
        const int tpr = 256 / R;
        const int chunk = (((E + tpr - 1) / tpr) + 3) & ~3;
        const int c_lo = min(part * chunk, E), c_hi = min(c_lo + chunk, E);
        float* my_row = s_logit + j * lstride;
        const bool work = hdr_ok && !*abort_flag;
        const float scale = ldexpf(1.0f, -hdr->scale_exp);
        if (nsplit == 1) named_bar_sync(1, 256);  // rows written by warps 2-5
        // pass 1: full logits (slices added in rank order), kept in slot 0,
        // and the K largest by logit -- the softmax is monotone in the
        // logit, so this is the probability order.  Experts arrive in
        // ascending index; one enters the list only when strictly larger
        // than the current K-th, so equal logits keep the lower index first
        // (the reference's repeated-argmax order).
        float bv[K];
        int bi[K];
#pragma unroll
        for (int k = 0; k < K; ++k) {
            bv[k] = -INFINITY;
            bi[k] = 0;
        }
        if (work) {
            for (int c = c_lo; c < c_hi; c += 4) {
                float4 l = *reinterpret_cast<const float4*>(my_row + c);
                for (int sl = 1; sl < nsplit; ++sl) {
                    const float4 o = *reinterpret_cast<const float4*>(my_row + sl * slot_floats + c);
                    l.x += o.x;
                    l.y += o.y;
                    l.z += o.z;
                    l.w += o.w;
                }
                const float lv[4] = {l.x * scale, l.y * scale, l.z * scale, l.w * scale};
                *reinterpret_cast<float4*>(my_row + c) = make_float4(lv[0], lv[1], lv[2], lv[3]);
#pragma unroll
                for (int q = 0; q < 4; ++q)
                    if (c + q < c_hi && lv[q] > bv[K - 1]) topk_insert<K>(bv, bi, lv[q], c + q);
            }
        }
        if (part) {
#pragma unroll
            for (int k = 0; k < K; ++k) {
                ctl->merge_v[et][k] = bv[k];
                ctl->merge_i[et][k] = bi[k];
            }
        }
        named_bar_sync(1, 256);
        if (!part) {
            // each later range's experts all follow the earlier ones', and
            // its list is in insertion order, so inserting the lists in
            // range order keeps ties ordered by index
            for (int pp = 1; pp < tpr; ++pp) {
                const int src = pp * R + j;
#pragma unroll
                for (int k = 0; k < K; ++k) {
                    const float v = ctl->merge_v[src][k];
                    if (v > bv[K - 1]) topk_insert<K>(bv, bi, v, ctl->merge_i[src][k]);
                }
            }
            ctl->row_max[j] = bv[0];
        }
        named_bar_sync(1, 256);
        // pass 2: sum of exponentials, each range in ascending expert order
        const float mx = ctl->row_max[j];
        float sum = 0.f;
        if (work) {
            for (int c = c_lo; c < c_hi; c += 4) {
                const float4 l = *reinterpret_cast<const float4*>(my_row + c);
                const float e4[4] = {expf(l.x - mx), expf(l.y - mx), expf(l.z - mx), expf(l.w - mx)};
#pragma unroll
                for (int q = 0; q < 4; ++q)
                    if (c + q < c_hi) sum += e4[q];
            }
        }
        ctl->merge_f[et] = sum;
        named_bar_sync(1, 256);
        const int t = row0 + int(crank) * R + j;
        if (!part && work && t < T) {
            sum = 0.f;
            for (int pp = 0; pp < tpr; ++pp) sum += ctl->merge_f[pp * R + j];
#pragma unroll
            for (int k = 0; k < K; ++k) {
                assignments[int64_t(t) * K + k] = bi[k];
                weights[int64_t(t) * K + k] = expf(bv[k] - mx) / sum;
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) {
        __syncwarp();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ncols) : "memory");
    }
}

using RouteKernel = void (*)(CUtensorMap, CUtensorMap, const RouterHeader*, int, int, int, int, int, int, int,
                            uint32_t, int32_t*, float*, uint32_t*);

template <int DT>
RouteKernel route_kernel_k(int K) {
    switch (K) {
        case 1: return route_kernel<DT, 1>;
        case 2: return route_kernel<DT, 2>;
        case 3: return route_kernel<DT, 3>;
        case 4: return route_kernel<DT, 4>;
        case 5: return route_kernel<DT, 5>;
        case 6: return route_kernel<DT, 6>;
        case 7: return route_kernel<DT, 7>;
        default: return route_kernel<DT, 8>;
    }
}
RouteKernel route_kernel_for(int dtype, int K) {
    return dtype == MOE_B200_BF16 ? route_kernel_k<MOE_B200_BF16>(K) : route_kernel_k<MOE_B200_F16>(K);
}

int sm_count_rt() {
    int dev = 0, n = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n > 0 ? n : 148;
}

int check_shape(const char* who, int d, int E, int dtype) {
    if (dtype != MOE_B200_F16 && dtype != MOE_B200_BF16)
        return fail(MOE_B200_ERR_INVALID_ARG, "%s: dtype %d is neither F16 nor BF16", who, dtype);
    if (d < 8 || d % 8 != 0) return fail(MOE_B200_ERR_UNSUPPORTED, "%s: d=%d must be a positive multiple of 8", who, d);
    const int emax = dtype == MOE_B200_BF16 ? 128 : 256;
    if (E < 1 || E > emax)
        return fail(MOE_B200_ERR_UNSUPPORTED, "%s: E=%d outside [1, %d] for this dtype", who, E, emax);
    return MOE_B200_OK;
}

}  // namespace
}  // namespace moe_b200

using namespace moe_b200;

extern "C" size_t moe_b200_router_weights_bytes(int d, int E, int dtype) {
    if (d < 1 || E < 1 || (dtype != MOE_B200_F16 && dtype != MOE_B200_BF16)) return 0;
    return kRouterHeaderBytes + size_t(pieces_for(dtype)) * round_up16(E) * size_t(d) * 2;
}

extern "C" int moe_b200_router_prepare(const float* w_gate, int d, int E, int dtype, void* packed_weights,
                                       void* stream) {
    if (int st = check_shape("router_prepare", d, E, dtype)) return st;
    if (!w_gate || !packed_weights) return fail(MOE_B200_ERR_INVALID_ARG, "router_prepare: null pointer");
    if (reinterpret_cast<uintptr_t>(packed_weights) % 16 != 0)
        return fail(MOE_B200_ERR_INVALID_ARG, "router_prepare: packed_weights must be 16-byte aligned");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int E_pad = round_up16(E), P = pieces_for(dtype);
    RouterHeader h = {};
    h.magic = 0;  // set by the split kernel once the pieces are written
    h.d = d;
    h.E = E;
    h.E_pad = E_pad;
    h.pieces = P;
    h.dtype = dtype;
    auto* hdr = static_cast<RouterHeader*>(packed_weights);
    cudaError_t err = cudaMemcpyAsync(hdr, &h, sizeof(h), cudaMemcpyHostToDevice, s);
    if (err != cudaSuccess) return cuda_fail(err, "router_prepare header");
    const int64_t n = int64_t(d) * E;
    const int blocks = int(std::min<int64_t>((n + 255) / 256, 1024));
    router_absmax_kernel<<<blocks, 256, 0, s>>>(w_gate, n, hdr);
    uint16_t* out = reinterpret_cast<uint16_t*>(static_cast<char*>(packed_weights) + kRouterHeaderBytes);
    const dim3 grid((d + 31) / 32, (E_pad + 31) / 32), block(32, 8);
    if (dtype == MOE_B200_BF16)
        router_split_kernel<MOE_B200_BF16><<<grid, block, 0, s>>>(w_gate, d, E, E_pad, hdr, out);
    else
        router_split_kernel<MOE_B200_F16><<<grid, block, 0, s>>>(w_gate, d, E, E_pad, hdr, out);
    err = cudaGetLastError();
    if (err != cudaSuccess) return cuda_fail(err, "router_prepare launch");
    // The host header copy must not outlive its stack frame before it ran.
    err = cudaStreamSynchronize(s);
    return err == cudaSuccess ? MOE_B200_OK : cuda_fail(err, "router_prepare");
}

extern "C" int moe_b200_route(const void* emb, int T, int d, int E, int K, int dtype, const void* packed_weights,
                              int32_t* assignments, float* weights, void* stream) {
    if (int st = check_shape("route", d, E, dtype)) return st;
    if (T < 0) return fail(MOE_B200_ERR_INVALID_ARG, "route: T=%d < 0", T);
    if (K < 1 || K > 8 || K > E) return fail(MOE_B200_ERR_UNSUPPORTED, "route: K=%d outside [1, min(8, E)]", K);
    if (!emb || !packed_weights || !assignments || !weights)
        return fail(MOE_B200_ERR_INVALID_ARG, "route: null pointer");
    if ((reinterpret_cast<uintptr_t>(emb) | reinterpret_cast<uintptr_t>(packed_weights)) % 16 != 0)
        return fail(MOE_B200_ERR_INVALID_ARG, "route: emb and packed_weights must be 16-byte aligned");
    if (T == 0) return MOE_B200_OK;
    uint32_t* st = device_status_word();
    if (!st) return fail(MOE_B200_ERR_CUDA, "route: device status word unavailable");
    const int E_pad = round_up16(E), P = pieces_for(dtype);
    const uint32_t sb = stage_bytes(E_pad, P);
    const int stages = int(std::min<size_t>(kRtMaxStages, kRtStageBudget / sb));
    if (stages < 2) return fail(MOE_B200_ERR_UNSUPPORTED, "route: E=%d does not fit two pipeline stages", E);
    const size_t slot_bytes = size_t(kRtTileM) * (E_pad + 4) * 4;
    const char* pieces = static_cast<const char*>(packed_weights) + kRouterHeaderBytes;
    CUtensorMap mx, mw;
    if (!make_map(&mx, emb, T, d, kRtTileM, dtype) || !make_map(&mw, pieces, int64_t(P) * E_pad, d, E_pad, dtype))
        return fail(MOE_B200_ERR_CUDA, "route: cuTensorMapEncodeTiled failed");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const auto* hdr = static_cast<const RouterHeader*>(packed_weights);
    const int tiles = (T + kRtTileM - 1) / kRtTileM;
    const int nk = (d + kRtTileK - 1) / kRtTileK;
    // Split the d features over a cluster of 2 or 4 CTAs per token tile when
    // the tiles alone cannot fill the SMs.  Each CTA then finishes 128 /
    // nsplit of the tile's rows and holds nsplit slices of them: 128 logit
    // rows whatever nsplit.
    int nsplit = 1;
    while (nsplit < 4 && tiles * nsplit * 2 <= sm_count_rt() && nsplit * 2 <= nk) nsplit *= 2;
    const size_t area = std::max(size_t(stages) * sb, slot_bytes);
    if (area > kRtStageBudget)
        return fail(MOE_B200_ERR_UNSUPPORTED, "route: E=%d logit rows exceed shared memory", E);
    const size_t smem = 1024 + area + sizeof(RouteSmem);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(tiles * nsplit);
    cfg.blockDim = dim3(kRtThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    if (nsplit > 1) {
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = nsplit;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    auto kern = route_kernel_for(dtype, K);
    cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (err == cudaSuccess)
        err = cudaLaunchKernelEx(&cfg, kern, mx, mw, hdr, T, d, E, E_pad, P, stages, nsplit, uint32_t(area),
                                 assignments, weights, st);
    return err == cudaSuccess ? MOE_B200_OK : cuda_fail(err, "route launch");
}
