// grouped_ffn.cu -- grouped SwiGLU expert FFN on the 5th-generation tensor
// cores (tcgen05 + TMEM, TMA-fed), sm_100a.
//
//   h[r, :] = silu(x[r] . Wg[e]^T) * (x[r] . Wu[e]^T)     (GEMM 1, K = d)
//   y[r, :] = h[r] . Wd[e]^T                               (GEMM 2, K = I)
// for every packed row r of segment s, e = expert of s; fp32 accumulation in
// TMEM, h and y rounded once to 16 bits.
//
// Replaces the reference's per-expert cublasHgemm loop (apps/bench_e2e.cu:
// 274-301, apps/bench_prefill.cu:854-884) and its CUTLASS sm80 GemmGrouped
// (apps/bench_prefill.cu:68-202, 812-852), both of which need the expert
// counts on the host; here the tile list is derived on the device from the
// segment offsets the packing kernel wrote.  The reference FFN has no
// activation; this one is SwiGLU (gate, up, down).
//
// One persistent kernel, one CTA per SM, 6 warps:
//   warp 0     TMA producer: A tile (128 rows x 64 K) + B tile per stage,
//              128-byte swizzle
//   warp 1     allocates TMEM (512 columns = two 128x256 fp32 accumulators)
//              and issues tcgen05.mma (N=256, K=16) from one lane
//   warps 2-5  epilogue: tcgen05.ld of their 32-lane quadrant, SwiGLU or
//              plain conversion, 16-byte stores
// Two CTA-group variants share the code:
//   CG=1  one SM per 128 x 256 tile, B tile of 256 rows, 4 stages
//   CG=2  (default) an SM pair (cluster of 2) per 256 x 256 tile:
//         tcgen05.mma.cta_group::2 with M=256 issued by the pair leader,
//         each CTA loading its own 128 A rows and half of the B rows, so
//         each SM stages 32 KB per K step instead of 48 KB and keeps 6
//         stages in flight; the TMA of both CTAs completes on the leader's
//         barrier, MMA completion is committed to both CTAs' barriers, and
//         the epilogue warps of both CTAs release the accumulator to the
//         leader.
// Tiles are (segment, row block, N block), N fastest, so concurrent CTAs
// share the A block and the expert's weights in L2.  Every wait is bounded;
// on expiry the CTA records MOE_B200_DEV_WAIT_TIMEOUT, raises a CTA-wide abort
// flag so the other roles stop waiting, and still frees its TMEM.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdlib>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "tcgen05.cuh"

namespace moe_b200 {

constexpr int kTileM = 128;
constexpr int kTileN = 256;
constexpr int kTileK = 64;  // 64 x 16-bit = one 128-byte swizzle row
constexpr int kFfnThreads = 192;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kABytes = kTileM * kTileK * 2;  // 16 KB: one CTA's A rows per stage
// Per-CTA stage geometry for CTA group CG (1: one SM per tile; 2: an SM pair
// computes a 256-row tile with tcgen05.mma.cta_group::2, each CTA holding
// 128 rows of A and half of the 256 B rows).
template <int CG> struct Geo {
    static constexpr int kBRows = kTileN / CG;                 // B rows held per CTA
    static constexpr uint32_t kBBytes = kBRows * kTileK * 2;   // 32 KB / 16 KB
    static constexpr int kStages = CG == 1 ? 4 : 6;            // 192 KB either way
    static constexpr int kBlockRows = kTileM * CG;             // rows per tile
};
constexpr int kMaxStages = 6;
constexpr int kMaxSegments = 1024;  // keeps shared memory under 227 KB

enum { kEpiSwiGLU = 0, kEpiStore = 1 };

// --- CTA pair (cluster of 2) helpers ---
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_id_x() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t num_clusters_x() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Shared::cluster address of the same shared variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_to_rank(const void* p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
    return r;
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ void umma_f16_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Completion of this thread's pair MMAs arrives on the barrier at a
// shared::cluster address (either CTA of the pair).
__device__ __forceinline__ void umma_commit_pair(uint32_t cluster_bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(cluster_bar)
                 : "memory");
}
// Pair TMA load into this CTA's shared memory, completing on the barrier at
// a shared::cluster address (the pair leader's).
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map, int x, int y,
                                                uint32_t cluster_bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(cluster_bar)
        : "memory");
}

// ------------------------------------------------------------ helpers -----

template <int DT>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
    if (DT == MOE_B200_BF16) {
        __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&v);
    } else {
        __half2 v = __floats2half2_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&v);
    }
}

__device__ __forceinline__ float silu(float g) { return g / (1.0f + __expf(-g)); }

struct FfnSmem {
    uint64_t full[kMaxStages];
    uint64_t empty[kMaxStages];
    uint64_t tmem_full[2];
    uint64_t tmem_empty[2];
    uint32_t tmem_base;
    int abort_flag;
    int nseg;
    int total_blocks;
};

// Epilogue staging: each epilogue warp owns 32 rows x 128 bytes (64 16-bit
// columns) of shared memory.  Lane r writes its accumulator row r; the 16-byte
// chunk j of row r sits at slot j ^ (r & 7), so that both the row-wise writes
// (8 lanes cover all 32 banks) and the chunk-wise reads are conflict-free.
constexpr uint32_t kWarpStageBytes = 32 * 128;
constexpr uint32_t kStageBytes = 4 * kWarpStageBytes;

__device__ __forceinline__ void stage_put(unsigned char* stg, int row, int chunk, const uint4& v) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(smem_u32(stg + row * 128 + ((chunk ^ (row & 7)) << 4))),
                 "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}

// Writes the warp's staged 32 x 64 columns to its rows 0..nrows-1 (columns
// col0 .. col0+63, clipped at n_out): 4 rows x 128 contiguous bytes per warp
// store instruction instead of 32 scattered 16-byte pieces.  Row r goes to
// dst + r * stride, or, when lane_row is given (scatter mode), to the row
// address lane r holds in lane_row.
__device__ __forceinline__ void stage_flush(const unsigned char* stg, int lane, uint16_t* dst, int64_t stride,
                                            int nrows, int col0, int n_out, uint16_t* lane_row) {
    __syncwarp();
    const int ch = lane & 7;
    const bool col_ok = col0 + ch * 8 < n_out;
#pragma unroll
    for (int it = 0; it < 8; ++it) {
        const int r = it * 4 + (lane >> 3);
        uint4 v;
        asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                     : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                     : "r"(smem_u32(stg + r * 128 + ((ch ^ (r & 7)) << 4)))
                     : "memory");
        uint16_t* row = dst ? dst + int64_t(r) * stride
                            : reinterpret_cast<uint16_t*>(__shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(lane_row), r));
        if (r < nrows && col_ok) st_v4(reinterpret_cast<uint4*>(row + col0) + ch, v);
    }
    __syncwarp();
}

// Rows that other ranks store into this GPU's memory (the expert-parallel
// receive buffer): before the first TMA load of a segment >= wait_seg0, the
// producer thread waits (bounded by one deadline) until every sender's data
// flag reached the epoch, then orders its TMA reads after that acquire.  On
// a timeout it records MOE_B200_DEV_WAIT_TIMEOUT and goes on.
__device__ __forceinline__ void wait_rows_once(const EpWait& w, bool& ready, uint32_t* dev_status) {
    if (ready) return;
    ready = true;
    const uint64_t t0 = globaltimer_ns();
    for (int i = 0; i < w.n; ++i) {
        while (ld_acquire_sys(w.flags + i) < w.epoch) {
            if (globaltimer_ns() - t0 > w.timeout_ns) {
                atomicOr(dev_status, MOE_B200_DEV_WAIT_TIMEOUT);
                i = w.n;
                break;
            }
            __nanosleep(64);
        }
    }
    fence_proxy_async_global();
}

// Maps a linear 128-row block index to (segment, block within segment).
__device__ __forceinline__ int find_segment(const int32_t* blk_prefix, int nseg, int g) {
    int lo = 0, hi = nseg - 1;
    while (lo < hi) {
        int mid = (lo + hi + 1) >> 1;
        if (blk_prefix[mid] <= g) lo = mid;
        else hi = mid - 1;
    }
    return lo;
}

// EPI = kEpiSwiGLU: B rows of N block n are gate rows [n*128, n*128+128) and up
// rows [I + n*128, ...) of the expert; the output has n_out = I columns.
// EPI = kEpiStore: B rows [n*256, n*256+256) of the expert; n_out columns.
template <int EPI, int DT, int CG>
__global__ void __launch_bounds__(kFfnThreads, 1)
grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                    const int32_t* __restrict__ seg_start, const int32_t* __restrict__ seg_expert,
                    int nseg, int kdim, int b_rows_per_expert, int n_out, int n_blocks,
                    int gate_up_split, uint16_t* __restrict__ out, int64_t out_stride,
                    uint32_t* __restrict__ dev_status, char* const* __restrict__ dst_base,
                    const int64_t* __restrict__ row_ret, const int32_t* __restrict__ gather_rows,
                    int gather_limit, EpSignal sig, EpWait rows_wait, int wait_seg0) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    // 1024-byte aligned stage buffers (SW128 atoms), control block after them.
    unsigned char* base = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    using GEO = Geo<CG>;
    constexpr int kStages = GEO::kStages;
    constexpr uint32_t kBBytes = GEO::kBBytes;
    constexpr int kBlockRows = GEO::kBlockRows;
    unsigned char* sA = base;
    unsigned char* sB = base + kStages * kABytes;
    unsigned char* s_stage = sB + kStages * kBBytes;            // epilogue staging, kStageBytes
    FfnSmem* ctl = reinterpret_cast<FfnSmem*>(s_stage + kStageBytes);
    int32_t* blk_prefix = reinterpret_cast<int32_t*>(ctl + 1);  // [nseg + 1]
    int32_t* s_start = blk_prefix + (nseg + 1);                 // [nseg + 1] row offsets
    // [nseg] expert of each segment.  In scatter mode (dst_base != nullptr)
    // row i of the input (the receive buffer) is stored at row
    // (row_ret[i] & 0xffffffff) of dst_base[row_ret[i] >> 32] -- the back
    // buffer of the rank that sent it, at its packed position there
    int32_t* s_exp = s_start + (nseg + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    volatile int* abort_flag = &ctl->abort_flag;
    // CTA-pair coordinates (CG = 2): rank 0 is the leader that issues the MMAs.
    const uint32_t crank = CG == 2 ? cluster_rank() : 0u;
    const int tile0 = CG == 2 ? int(cluster_id_x()) : int(blockIdx.x);
    const int tile_step = CG == 2 ? int(num_clusters_x()) : int(gridDim.x);

    // Set-up: barriers, block prefix over segments, TMEM.
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&ctl->full[s], 1);
            mbar_init(&ctl->empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&ctl->tmem_full[b], 1);
            mbar_init(&ctl->tmem_empty[b], 4 * CG);  // epilogue warps of every CTA of the group
        }
        ctl->abort_flag = 0;
        mbar_fence_init();
    }
    if (warp == 0) {
        // blk_prefix[i] = row blocks of the segments before segment i
        int run = 0;
        for (int s0 = 0; s0 < nseg; s0 += 32) {
            int i = s0 + lane;
            int cnt = 0;
            if (i < nseg) {
                const int lo = seg_start[i];
                s_start[i] = lo;
                s_exp[i] = seg_expert ? seg_expert[i] : i;
                const int rows = seg_start[i + 1] - lo;
                cnt = rows > 0 ? (rows + kBlockRows - 1) / kBlockRows : 0;
            }
            int incl = cnt;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                int v = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += v;
            }
            if (i < nseg) blk_prefix[i] = run + incl - cnt;
            run += __shfl_sync(0xffffffffu, incl, 31);
        }
        if (lane == 0) {
            blk_prefix[nseg] = run;
            s_start[nseg] = seg_start[nseg];
            ctl->total_blocks = run;
        }
        if (lane == 0) {
            prefetch_tmap(&tmap_a);
            prefetch_tmap(&tmap_b);
        }
    }
    if (warp == 1) {
        if (CG == 1) {
            asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                             smem_u32(&ctl->tmem_base)),
                         "r"(kTmemCols)
                         : "memory");
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
        } else {
            asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                             smem_u32(&ctl->tmem_base)),
                         "r"(kTmemCols)
                         : "memory");
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
        }
    }
    tc_fence_before();
    __syncthreads();
    if (CG == 2) cluster_sync();  // both CTAs' barriers initialised before any cross-CTA signal
    tc_fence_after();

    const uint32_t tmem = ctl->tmem_base;
    const int total_tiles = ctl->total_blocks * n_blocks;
    const int nk = (kdim + kTileK - 1) / kTileK;
    const uint32_t leader_full0 = CG == 2 ? map_to_rank(&ctl->full[0], 0) : 0u;

    if (warp == 0 && CG == 1 && gather_rows) {
        // ---------------- TMA producer, gathered A rows ----------------
        // Row i of a tile is token gather_rows[packed row]: each lane fetches
        // 4 of the 128 rows per K step with one tile::gather4 load (a 1-row
        // box of 64 columns; the 4 rows land as 512 contiguous bytes of the
        // 128-byte-swizzled tile), lane 0 arms the barrier and loads B.
        uint32_t it = 0;
        bool rows_ready = rows_wait.flags == nullptr;
        const int total_rows = s_start[nseg];
        for (int tile = tile0; tile < total_tiles && !*abort_flag; tile += tile_step) {
            const int g = tile / n_blocks, n = tile % n_blocks;
            const int s = find_segment(blk_prefix, nseg, g);
            const int e = s_exp[s];
            if (s >= wait_seg0) wait_rows_once(rows_wait, rows_ready, dev_status);  // every lane issues loads
            const int row0 = s_start[s] + (g - blk_prefix[s]) * kBlockRows;
            int r4[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int p = row0 + lane * 4 + q;  // rows past the segment are masked in the epilogue
                const int t = p < total_rows ? __ldg(gather_rows + p) : 0;
                r4[q] = (t >= 0 && t < gather_limit) ? t : 0;
            }
            bool ok = true;
            for (int kb = 0; kb < nk; ++kb, ++it) {
                const int st = int(it % kStages);
                if (lane == 0)
                    ok = wait_or_abort(&ctl->empty[st], ((it / kStages) & 1u) ^ 1u, abort_flag, dev_status);
                if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) break;
                if (lane == 0) mbar_arrive_expect_tx(&ctl->full[st], kABytes + kBBytes);
                __syncwarp();
                tma_gather4(sA + st * kABytes + lane * 512, &tmap_a, kb * kTileK, r4[0], r4[1], r4[2], r4[3],
                            &ctl->full[st]);
                if (lane == 0) {
                    unsigned char* b = sB + st * kBBytes;
                    if (EPI == kEpiSwiGLU) {
                        const int brow = e * b_rows_per_expert + n * (kTileN / 2);
                        tma_load_2d(b, &tmap_b, kb * kTileK, brow, &ctl->full[st]);
                        tma_load_2d(b + kBBytes / 2, &tmap_b, kb * kTileK, brow + gate_up_split, &ctl->full[st]);
                    } else {
                        tma_load_2d(b, &tmap_b, kb * kTileK, e * b_rows_per_expert + n * kTileN, &ctl->full[st]);
                    }
                }
            }
            if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) break;
        }
        if (lane == 0 && *abort_flag) drain_stages(ctl->full, it, kStages);
    } else if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            uint32_t it = 0;
            bool rows_ready = rows_wait.flags == nullptr;
            for (int tile = tile0; tile < total_tiles && !*abort_flag; tile += tile_step) {
                const int g = tile / n_blocks, n = tile % n_blocks;
                const int s = find_segment(blk_prefix, nseg, g);
                const int e = s_exp[s];
                if (s >= wait_seg0) wait_rows_once(rows_wait, rows_ready, dev_status);
                const int row0 = s_start[s] + (g - blk_prefix[s]) * kBlockRows + int(crank) * kTileM;
                for (int kb = 0; kb < nk; ++kb, ++it) {
                    const int st = int(it % kStages);
                    if (!wait_or_abort(&ctl->empty[st], ((it / kStages) & 1u) ^ 1u, abort_flag, dev_status))
                        break;
                    unsigned char* b = sB + st * kBBytes;
                    if (CG == 1) {
                        mbar_arrive_expect_tx(&ctl->full[st], kABytes + kBBytes);
                        tma_load_2d(sA + st * kABytes, &tmap_a, kb * kTileK, row0, &ctl->full[st]);
                        if (EPI == kEpiSwiGLU) {
                            const int brow = e * b_rows_per_expert + n * (kTileN / 2);
                            tma_load_2d(b, &tmap_b, kb * kTileK, brow, &ctl->full[st]);
                            tma_load_2d(b + kBBytes / 2, &tmap_b, kb * kTileK, brow + gate_up_split,
                                        &ctl->full[st]);
                        } else {
                            tma_load_2d(b, &tmap_b, kb * kTileK, e * b_rows_per_expert + n * kTileN,
                                        &ctl->full[st]);
                        }
                    } else {
                        // Both CTAs load their halves; the bytes land on the leader's barrier,
                        // which the leader arms with the pair's total.
                        const uint32_t fbar = leader_full0 + uint32_t(st) * 8u;
                        if (crank == 0) mbar_arrive_expect_tx(&ctl->full[st], 2 * (kABytes + kBBytes));
                        tma_load_2d_pair(sA + st * kABytes, &tmap_a, kb * kTileK, row0, fbar);
                        const int brow = EPI == kEpiSwiGLU
                                             ? e * b_rows_per_expert + n * (kTileN / 2) + int(crank) * gate_up_split
                                             : e * b_rows_per_expert + n * kTileN + int(crank) * (kTileN / 2);
                        tma_load_2d_pair(b, &tmap_b, kb * kTileK, brow, fbar);
                    }
                }
            }
            // the pair's loads complete on the leader's barriers; the final
            // cluster barrier keeps the peer resident until the leader drained
            if (crank == 0 && *abort_flag) drain_stages(ctl->full, it, kStages);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer (the pair leader for CG = 2) ----------------
        if (lane == 0 && crank == 0) {
            const uint32_t idesc = umma_idesc_mn(DT == MOE_B200_BF16 ? 1 : 0, kBlockRows, kTileN);
            uint32_t it = 0, j = 0;
            for (int tile = tile0; tile < total_tiles && !*abort_flag; tile += tile_step, ++j) {
                const int buf = int(j & 1u);
                if (!wait_or_abort(&ctl->tmem_empty[buf], ((j >> 1) & 1u) ^ 1u, abort_flag, dev_status))
                    break;
                tc_fence_after();
                const uint32_t d_tmem = tmem + uint32_t(buf) * kTileN;
                bool ok = true;
                for (int kb = 0; kb < nk; ++kb, ++it) {
                    const int st = int(it % kStages);
                    if (!wait_or_abort(&ctl->full[st], (it / kStages) & 1u, abort_flag, dev_status)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(sA + st * kABytes);
                    const uint32_t b_addr = smem_u32(sB + st * kBBytes);
#pragma unroll
                    for (int kk = 0; kk < kTileK / 16; ++kk) {
                        // +32 bytes per 16-element K step inside the 128-byte swizzle row
                        const uint64_t ad = umma_desc_sw128(a_addr + kk * 32), bd = umma_desc_sw128(b_addr + kk * 32);
                        const uint32_t acc = (kb > 0 || kk > 0) ? 1u : 0u;
                        if (CG == 1) umma_f16(d_tmem, ad, bd, idesc, acc);
                        else umma_f16_pair(d_tmem, ad, bd, idesc, acc);
                    }
                    if (CG == 1) {
                        umma_commit(&ctl->empty[st]);
                    } else {  // free the stage in both CTAs
                        umma_commit_pair(map_to_rank(&ctl->empty[st], 0));
                        umma_commit_pair(map_to_rank(&ctl->empty[st], 1));
                    }
                }
                if (!ok) break;
                if (CG == 1) {
                    umma_commit(&ctl->tmem_full[buf]);
                } else {
                    umma_commit_pair(map_to_rank(&ctl->tmem_full[buf], 0));
                    umma_commit_pair(map_to_rank(&ctl->tmem_full[buf], 1));
                }
            }
        }
    } else {
        // ---------------- epilogue (warps 2..5) ----------------
        const int quad = warp & 3;  // TMEM lanes 32*quad .. 32*quad+31
        unsigned char* stg = s_stage + quad * kWarpStageBytes;
        uint32_t j = 0;
        const uint32_t leader_tmem_empty0 = CG == 2 ? map_to_rank(&ctl->tmem_empty[0], 0) : 0u;
        for (int tile = tile0; tile < total_tiles; tile += tile_step, ++j) {
            const int buf = int(j & 1u);
            if (!wait_or_abort(&ctl->tmem_full[buf], (j >> 1) & 1u, abort_flag, dev_status)) break;
            tc_fence_after();
            const int g = tile / n_blocks, n = tile % n_blocks;
            const int s = find_segment(blk_prefix, nseg, g);
            const int blk = g - blk_prefix[s];
            const int seg_rows = s_start[s + 1] - s_start[s];
            // This warp's 32 rows start at segment row w_row0; nrows_w of them are in the segment.
            const int w_row0 = blk * kBlockRows + int(crank) * kTileM + quad * 32;
            const int nrows_w = seg_rows - w_row0;
            // Destinations: consecutive rows of the local output, or in
            // scatter mode each row's own return address (lane r holds row r's).
            uint16_t* dst0 = dst_base ? nullptr : out + (int64_t(s_start[s]) + w_row0) * out_stride;
            uint16_t* lane_row = nullptr;
            if (dst_base && lane < nrows_w) {
                const int64_t rr = row_ret[int64_t(s_start[s]) + w_row0 + lane];
                lane_row = reinterpret_cast<uint16_t*>(dst_base[int(rr >> 32)]) + int64_t(uint32_t(rr)) * out_stride;
            }
            const uint32_t t_row = tmem + uint32_t(buf) * kTileN + (uint32_t(quad * 32) << 16);
            if (EPI == kEpiSwiGLU) {
                // 32 gate + 32 up columns per TMEM round trip; every second
                // round flushes 64 output columns from the staging tile.
#pragma unroll 1
                for (int c = 0; c < kTileN / 2; c += 32) {
                    uint32_t gr[2][16], ur[2][16];
                    tmem_ld16(t_row + c, gr[0]);
                    tmem_ld16(t_row + c + 16, gr[1]);
                    tmem_ld16(t_row + kTileN / 2 + c, ur[0]);
                    tmem_ld16(t_row + kTileN / 2 + c + 16, ur[1]);
                    tmem_wait_ld();
#pragma unroll
                    for (int hb = 0; hb < 2; ++hb) {
                        uint32_t o[8];
#pragma unroll
                        for (int q = 0; q < 8; ++q) {
                            const float g0 = __uint_as_float(gr[hb][2 * q]), g1 = __uint_as_float(gr[hb][2 * q + 1]);
                            const float u0 = __uint_as_float(ur[hb][2 * q]), u1 = __uint_as_float(ur[hb][2 * q + 1]);
                            o[q] = pack2<DT>(silu(g0) * u0, silu(g1) * u1);
                        }
                        const int ch = ((c & 32) >> 3) + 2 * hb;  // 16-byte chunk of the 64-column staging row
                        stage_put(stg, lane, ch, make_uint4(o[0], o[1], o[2], o[3]));
                        stage_put(stg, lane, ch + 1, make_uint4(o[4], o[5], o[6], o[7]));
                    }
                    if (c & 32)
                        stage_flush(stg, lane, dst0, out_stride, nrows_w, n * (kTileN / 2) + c - 32, n_out, lane_row);
                }
            } else {
                // 64 columns per TMEM round trip
#pragma unroll 1
                for (int c = 0; c < kTileN; c += 64) {
                    uint32_t v[4][16];
#pragma unroll
                    for (int q4 = 0; q4 < 4; ++q4) tmem_ld16(t_row + c + 16 * q4, v[q4]);
                    tmem_wait_ld();
#pragma unroll
                    for (int q4 = 0; q4 < 4; ++q4) {
                        uint32_t o[8];
#pragma unroll
                        for (int q = 0; q < 8; ++q)
                            o[q] = pack2<DT>(__uint_as_float(v[q4][2 * q]), __uint_as_float(v[q4][2 * q + 1]));
                        stage_put(stg, lane, 2 * q4, make_uint4(o[0], o[1], o[2], o[3]));
                        stage_put(stg, lane, 2 * q4 + 1, make_uint4(o[4], o[5], o[6], o[7]));
                    }
                    stage_flush(stg, lane, dst0, out_stride, nrows_w, n * kTileN + c, n_out, lane_row);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if (CG == 1) mbar_arrive(&ctl->tmem_empty[buf]);
                else mbar_arrive_cluster(leader_tmem_empty0 + uint32_t(buf) * 8u);
            }
        }
    }

    // Stores to another GPU's memory must be visible system-wide before the
    // flag that announces them (raised by a later kernel in this stream).
    if (dst_base && warp >= 2) __threadfence_system();
    tc_fence_before();
    __syncthreads();
    // expert parallel: the last CTA to finish raises the senders' back flags
    if (sig.peer && threadIdx.x == 0) ep_signal_done(sig, *abort_flag != 0);
    if (CG == 2) cluster_sync();  // no CTA leaves while its pair may still signal it
    tc_fence_after();
    if (warp == 1) {
        __syncwarp();
        if (CG == 1)
            asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols)
                         : "memory");
        else
            asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols)
                         : "memory");
    }
}

// ----------------------------------------------------------------- host ----

template <int CG>
static size_t ffn_smem_bytes(int nseg) {
    return 1024 + Geo<CG>::kStages * (kABytes + Geo<CG>::kBBytes) + kStageBytes + sizeof(FfnSmem) +
           size_t(3 * nseg + 2) * 4;
}

static int sm_count_ffn() {
    int dev = 0, n = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n > 0 ? n : 148;
}

// CTA groups of the two GEMMs, bit 0: gate/up GEMM on SM pairs, bit 1: down
// GEMM on SM pairs.  MOE_B200_FFN=1sm / 2sm forces one form for both; the
// default runs the gate/up GEMM on single SMs and the down GEMM (whose
// epilogue stores twice the columns per MMA step) on SM pairs when the
// segments average at least 512 rows, so that 256-row tiles waste little.
static int ffn_cta_groups(int rows, int nseg) {
    const char* v = std::getenv("MOE_B200_FFN");
    if (v && std::strcmp(v, "1sm") == 0) return 0;
    if (v && std::strcmp(v, "2sm") == 0) return 3;
    return rows >= 512 * nseg ? 2 : 0;
}

template <int EPI, int DT, int CG>
static cudaError_t launch_gemm(const CUtensorMap& ma, const CUtensorMap& mb_, const int32_t* seg_start,
                               const int32_t* seg_expert, int nseg, int rows, int kdim, int b_rows_per_expert,
                               int n_out, int n_blocks, int split, void* out, int64_t out_stride,
                               uint32_t* st, cudaStream_t stream, char* const* dst_base = nullptr,
                               const int64_t* row_ret = nullptr, const int32_t* gather_rows = nullptr,
                               int gather_limit = 0, const EpSignal* sig = nullptr,
                               const EpWait* rows_wait = nullptr, int wait_seg0 = 0) {
    EpSignal no_sig{};
    EpWait no_wait{};
    const size_t smem = ffn_smem_bytes<CG>(nseg);
    auto kern = grouped_gemm_kernel<EPI, DT, CG>;
    cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (err != cudaSuccess) return err;
    // Upper bound on tiles: every segment may add one partial block.
    const int64_t max_tiles = (int64_t(rows) / Geo<CG>::kBlockRows + nseg) * n_blocks;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = pdl_config(dim3(1), dim3(kFfnThreads), smem, stream);
    int groups = sm_count_ffn() / CG;
    if (CG == 2) {
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        cfg.gridDim = dim3(2 * groups);
        int active = 0;
        if (cudaOccupancyMaxActiveClusters(&active, kern, &cfg) == cudaSuccess && active > 0 && active < groups)
            groups = active;
        cudaGetLastError();
    }
    if (max_tiles < groups) groups = int(max_tiles > 0 ? max_tiles : 1);
    cfg.gridDim = dim3(CG * groups);
    return cudaLaunchKernelEx(&cfg, kern, ma, mb_, seg_start, seg_expert, nseg, kdim, b_rows_per_expert, n_out,
                              n_blocks, split, static_cast<uint16_t*>(out), out_stride, st, dst_base, row_ret,
                              gather_rows, gather_limit, sig ? *sig : no_sig, rows_wait ? *rows_wait : no_wait,
                              wait_seg0);
}

template <int DT>
static cudaError_t launch_ffn(int cg, const CUtensorMap& mx, const CUtensorMap& mwgu, const CUtensorMap& mh,
                              const CUtensorMap& mwd, const int32_t* seg_start, const int32_t* seg_expert, int nseg,
                              int rows, int d, int I, void* h, void* y, uint32_t* st, cudaStream_t s,
                              char* const* dst_base, const int64_t* row_ret, const int32_t* gather_rows,
                              int gather_T, const EpSignal* sig, const EpWait* rows_wait, int wait_seg0) {
    const int nb1 = (I + kTileN / 2 - 1) / (kTileN / 2);
    const int nb2 = (d + kTileN - 1) / kTileN;
    // The gathered form of GEMM 1 runs on single SMs.
    cudaError_t err =
        ((cg & 1) && !gather_rows)
            ? launch_gemm<kEpiSwiGLU, DT, 2>(mx, mwgu, seg_start, seg_expert, nseg, rows, d, 2 * I, I, nb1, I, h, I,
                                             st, s, nullptr, nullptr, nullptr, 0, nullptr, rows_wait, wait_seg0)
            : launch_gemm<kEpiSwiGLU, DT, 1>(mx, mwgu, seg_start, seg_expert, nseg, rows, d, 2 * I, I, nb1, I, h, I,
                                             st, s, nullptr, nullptr, gather_rows, gather_T, nullptr, rows_wait,
                                             wait_seg0);
    if (err != cudaSuccess) return err;
    return (cg & 2) ? launch_gemm<kEpiStore, DT, 2>(mh, mwd, seg_start, seg_expert, nseg, rows, I, d, d, nb2, 0, y, d,
                                                    st, s, dst_base, row_ret, nullptr, 0, sig)
                    : launch_gemm<kEpiStore, DT, 1>(mh, mwd, seg_start, seg_expert, nseg, rows, I, d, d, nb2, 0, y, d,
                                                    st, s, dst_base, row_ret, nullptr, 0, sig);
}

int fail(int code, const char* fmt, ...);
int cuda_fail(cudaError_t err, const char* where);

}  // namespace moe_b200

namespace moe_b200 {
int grouped_swiglu_impl(const void* x, const int32_t* seg_start, const int32_t* seg_expert, int nseg, int rows,
                        int d, int I, int E, const void* w_gate_up, const void* w_down, int dtype, void* h,
                        void* y, cudaStream_t s, char* const* dst_base, const int64_t* row_ret,
                        const int32_t* gather_rows, int gather_T, const EpSignal* sig, const EpWait* rows_wait,
                        int wait_seg0) {
    if (nseg < 1 || rows < 0 || d < 1 || I < 1 || E < 1)
        return fail(MOE_B200_ERR_INVALID_ARG, "grouped_swiglu: need nseg>=1, rows>=0, d>=1, I>=1, E>=1");
    if (nseg > kMaxSegments)
        return fail(MOE_B200_ERR_UNSUPPORTED, "grouped_swiglu: %d segments exceed %d", nseg, kMaxSegments);
    if (dtype != MOE_B200_F16 && dtype != MOE_B200_BF16)
        return fail(MOE_B200_ERR_INVALID_ARG, "grouped_swiglu: dtype %d is neither F16 nor BF16", dtype);
    if (d % 16 != 0 || I % 16 != 0)
        return fail(MOE_B200_ERR_UNSUPPORTED, "grouped_swiglu: d and I must be multiples of 16 (d=%d I=%d)", d, I);
    if (!x || !seg_start || !w_gate_up || !w_down || !h || (!y && !dst_base))
        return fail(MOE_B200_ERR_INVALID_ARG, "grouped_swiglu: null pointer");
    const uintptr_t al = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w_gate_up) |
                         reinterpret_cast<uintptr_t>(w_down) | reinterpret_cast<uintptr_t>(h) |
                         reinterpret_cast<uintptr_t>(y);
    if (dst_base && !row_ret)
        return fail(MOE_B200_ERR_INVALID_ARG, "grouped_swiglu: scatter mode needs the rows' return addresses");
    if (al % 16 != 0) return fail(MOE_B200_ERR_INVALID_ARG, "grouped_swiglu: pointers must be 16-byte aligned");
    if (rows == 0 && !sig) return MOE_B200_OK;
    uint32_t* st = device_status_word();
    if (!st) return fail(MOE_B200_ERR_CUDA, "grouped_swiglu: device status word unavailable");
    const int cg = ffn_cta_groups(rows, nseg);
    CUtensorMap mx, mwgu, mh, mwd;
    // A boxes hold one CTA's 128 rows; each CTA of a pair holds half of the
    // 256 B rows of a down-projection tile.
    // Gathered form: x holds gather_T token rows and packed row r is token
    // gather_rows[r] (a one-row box for tile::gather4); otherwise x is packed.
    if ((gather_rows && gather_T < 1) ||
        !make_map(&mx, x, gather_rows ? gather_T : rows, d, gather_rows ? 1 : kTileM, dtype) ||
        !make_map(&mwgu, w_gate_up, int64_t(E) * 2 * I, d, kTileN / 2, dtype) ||
        !make_map(&mh, h, rows, I, kTileM, dtype) ||
        !make_map(&mwd, w_down, int64_t(E) * d, I, (cg & 2) ? kTileN / 2 : kTileN, dtype))
        return fail(MOE_B200_ERR_CUDA, "grouped_swiglu: cuTensorMapEncodeTiled failed");
    const cudaError_t err =
        dtype == MOE_B200_BF16
            ? launch_ffn<MOE_B200_BF16>(cg, mx, mwgu, mh, mwd, seg_start, seg_expert, nseg, rows, d, I, h, y, st, s,
                                        dst_base, row_ret, gather_rows, gather_T, sig, rows_wait, wait_seg0)
            : launch_ffn<MOE_B200_F16>(cg, mx, mwgu, mh, mwd, seg_start, seg_expert, nseg, rows, d, I, h, y, st, s,
                                       dst_base, row_ret, gather_rows, gather_T, sig, rows_wait, wait_seg0);
    return err == cudaSuccess ? MOE_B200_OK : cuda_fail(err, "grouped_swiglu launch");
}
}  // namespace moe_b200

namespace moe_b200 {
// Activation-free grouped FFN (the reference's expert: up-projection, then
// down-projection, each result rounded once to 16 bits), on the same
// persistent tcgen05 kernel in its plain-store form:
//   mid[r] = x[r] . Wup[e]^T   (K = d, N = F)      y[r] = mid[r] . Wdown[e]^T   (K = F, N = d)
template <int DT>
static cudaError_t launch_plain_ffn(int cg, const CUtensorMap& mx, const CUtensorMap& mwu, const CUtensorMap& mmid,
                                    const CUtensorMap& mwd, const int32_t* seg_start, const int32_t* seg_expert,
                                    int nseg, int rows, int d, int F, void* mid, void* y, uint32_t* st,
                                    cudaStream_t s) {
    const int nb1 = (F + kTileN - 1) / kTileN;
    const int nb2 = (d + kTileN - 1) / kTileN;
    cudaError_t err = (cg & 1) ? launch_gemm<kEpiStore, DT, 2>(mx, mwu, seg_start, seg_expert, nseg, rows, d, F, F,
                                                              nb1, 0, mid, F, st, s)
                               : launch_gemm<kEpiStore, DT, 1>(mx, mwu, seg_start, seg_expert, nseg, rows, d, F, F,
                                                              nb1, 0, mid, F, st, s);
    if (err != cudaSuccess) return err;
    return (cg & 2) ? launch_gemm<kEpiStore, DT, 2>(mmid, mwd, seg_start, seg_expert, nseg, rows, F, d, d, nb2, 0, y,
                                                    d, st, s)
                    : launch_gemm<kEpiStore, DT, 1>(mmid, mwd, seg_start, seg_expert, nseg, rows, F, d, d, nb2, 0, y,
                                                    d, st, s);
}

int grouped_ffn_plain_impl(const void* x, const int32_t* seg_start, const int32_t* seg_expert, int nseg, int rows,
                           int d, int F, int E, const void* w_up, const void* w_down, int dtype, void* mid, void* y,
                           cudaStream_t s) {
    if (nseg < 1 || rows < 0 || d < 1 || F < 1 || E < 1)
        return fail(MOE_B200_ERR_INVALID_ARG, "grouped_ffn: need nseg>=1, rows>=0, d>=1, F>=1, E>=1");
    if (nseg > kMaxSegments)
        return fail(MOE_B200_ERR_UNSUPPORTED, "grouped_ffn: %d segments exceed %d", nseg, kMaxSegments);
    if (dtype != MOE_B200_F16 && dtype != MOE_B200_BF16)
        return fail(MOE_B200_ERR_INVALID_ARG, "grouped_ffn: dtype %d is neither F16 nor BF16", dtype);
    if (d % 16 != 0 || F % 16 != 0)
        return fail(MOE_B200_ERR_UNSUPPORTED, "grouped_ffn: d and F must be multiples of 16 (d=%d F=%d)", d, F);
    if (!x || !seg_start || !w_up || !w_down || !mid || !y)
        return fail(MOE_B200_ERR_INVALID_ARG, "grouped_ffn: null pointer");
    const uintptr_t al = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w_up) |
                         reinterpret_cast<uintptr_t>(w_down) | reinterpret_cast<uintptr_t>(mid) |
                         reinterpret_cast<uintptr_t>(y);
    if (al % 16 != 0) return fail(MOE_B200_ERR_INVALID_ARG, "grouped_ffn: pointers must be 16-byte aligned");
    if (rows == 0) return MOE_B200_OK;
    uint32_t* st = device_status_word();
    if (!st) return fail(MOE_B200_ERR_CUDA, "grouped_ffn: device status word unavailable");
    const int cg = ffn_cta_groups(rows, nseg);
    // B boxes: a CTA of an SM pair holds half of the 256 B rows of a tile
    CUtensorMap mx, mwu, mmid, mwd;
    if (!make_map(&mx, x, rows, d, kTileM, dtype) ||
        !make_map(&mwu, w_up, int64_t(E) * F, d, (cg & 1) ? kTileN / 2 : kTileN, dtype) ||
        !make_map(&mmid, mid, rows, F, kTileM, dtype) ||
        !make_map(&mwd, w_down, int64_t(E) * d, F, (cg & 2) ? kTileN / 2 : kTileN, dtype))
        return fail(MOE_B200_ERR_CUDA, "grouped_ffn: cuTensorMapEncodeTiled failed");
    const cudaError_t err =
        dtype == MOE_B200_BF16
            ? launch_plain_ffn<MOE_B200_BF16>(cg, mx, mwu, mmid, mwd, seg_start, seg_expert, nseg, rows, d, F, mid, y,
                                              st, s)
            : launch_plain_ffn<MOE_B200_F16>(cg, mx, mwu, mmid, mwd, seg_start, seg_expert, nseg, rows, d, F, mid, y,
                                             st, s);
    return err == cudaSuccess ? MOE_B200_OK : cuda_fail(err, "grouped_ffn launch");
}

// Per-expert transpose [E][R][C] -> [E][C][R] of 16-bit words through a
// 32 x 32 shared-memory tile (coalesced reads and writes): turns the
// reference's expert weights (W1 [E][d][F], W2 [E][F][d], row-major "B"
// operands of C = A . B) into the K-major w_up [E][F][d] / w_down [E][d][F].
__global__ void __launch_bounds__(256)
transpose_experts_kernel(const uint16_t* __restrict__ src, uint16_t* __restrict__ dst, int R, int C) {
    __shared__ uint16_t tile[32][33];
    const int e = blockIdx.z;
    const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
    const uint16_t* s = src + size_t(e) * R * C;
    uint16_t* o = dst + size_t(e) * R * C;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8 threads
    for (int j = ty; j < 32; j += 8) {
        const int r = r0 + j, c = c0 + tx;
        if (r < R && c < C) tile[j][tx] = s[size_t(r) * C + c];
    }
    __syncthreads();
    for (int j = ty; j < 32; j += 8) {
        const int c = c0 + j, r = r0 + tx;
        if (c < C && r < R) o[size_t(c) * R + r] = tile[tx][j];
    }
}

static cudaError_t launch_transpose_experts(const void* src, void* dst, int E, int R, int C, cudaStream_t s) {
    if (E < 1 || R < 1 || C < 1) return cudaSuccess;
    if (E > 65535) return cudaErrorInvalidValue;
    dim3 grid((C + 31) / 32, (R + 31) / 32, E);
    transpose_experts_kernel<<<grid, 256, 0, s>>>(static_cast<const uint16_t*>(src), static_cast<uint16_t*>(dst), R,
                                                   C);
    return cudaGetLastError();
}
}  // namespace moe_b200

extern "C" int moe_b200_grouped_ffn(const void* x, const int32_t* seg_start, const int32_t* seg_expert, int nseg,
                                    int rows, int d, int F, int E, const void* w_up, const void* w_down, int dtype,
                                    void* mid, void* y, void* stream) {
    return moe_b200::grouped_ffn_plain_impl(x, seg_start, seg_expert, nseg, rows, d, F, E, w_up, w_down, dtype, mid,
                                            y, static_cast<cudaStream_t>(stream));
}

extern "C" int moe_b200_ffn_weights_from_reference(const void* w1, const void* w2, int E, int d, int F, void* w_up,
                                                   void* w_down, void* stream) {
    using namespace moe_b200;
    if (!w1 || !w2 || !w_up || !w_down || E < 1 || d < 1 || F < 1)
        return fail(MOE_B200_ERR_INVALID_ARG, "ffn_weights_from_reference: need all buffers and E, d, F >= 1");
    if (E > 65535) return fail(MOE_B200_ERR_UNSUPPORTED, "ffn_weights_from_reference: E=%d above 65535", E);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t err = launch_transpose_experts(w1, w_up, E, d, F, s);        // [E][d][F] -> [E][F][d]
    if (err == cudaSuccess) err = launch_transpose_experts(w2, w_down, E, F, d, s);  // [E][F][d] -> [E][d][F]
    return err == cudaSuccess ? MOE_B200_OK : cuda_fail(err, "ffn_weights_from_reference launch");
}

extern "C" int moe_b200_grouped_swiglu(const void* x, const int32_t* seg_start, const int32_t* seg_expert,
                                       int nseg, int rows, int d, int I, int E, const void* w_gate_up,
                                       const void* w_down, int dtype, void* h, void* y, void* stream) {
    return moe_b200::grouped_swiglu_impl(x, seg_start, seg_expert, nseg, rows, d, I, E, w_gate_up, w_down, dtype,
                                         h, y, static_cast<cudaStream_t>(stream), nullptr, nullptr, nullptr, 0,
                                         nullptr, nullptr, 0);
}

extern "C" int moe_b200_grouped_swiglu_gather(const void* x_tokens, int T, const int32_t* row_token,
                                              const int32_t* seg_start, const int32_t* seg_expert, int nseg, int rows,
                                              int d, int I, int E, const void* w_gate_up, const void* w_down,
                                              int dtype, void* h, void* y, void* stream) {
    if (!row_token || T < 1)
        return moe_b200::fail(MOE_B200_ERR_INVALID_ARG, "grouped_swiglu_gather: need row_token and T >= 1");
    return moe_b200::grouped_swiglu_impl(x_tokens, seg_start, seg_expert, nseg, rows, d, I, E, w_gate_up, w_down,
                                         dtype, h, y, static_cast<cudaStream_t>(stream), nullptr, nullptr, row_token,
                                         T, nullptr, nullptr, 0);
}
