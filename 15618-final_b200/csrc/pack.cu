// pack.cu -- stable MoE token packing for sm_100a.
//
// Output contract: moe::cpu_scatter (reference src/common/cpu_reference.cpp:
// 12-51): rows grouped by expert, ascending (t, k) inside each expert,
// perm / packed_weights / expert_count / expert_start bit-identical.
//
// Two kernels, one stream, no CUB and no host round trip:
//
//  1. route_scan_kernel  (reads T*K*4 bytes of assignments)
//     One CTA per tile of slots, tiles claimed in order through an atomic
//     ticket so that every earlier tile is already running (forward progress
//     of the look-back).  Per tile: a warp-level __match_any_sync histogram
//     (pass 1), a per-expert prefix over the tile's warps, then a decoupled
//     look-back across tiles, one thread per expert, that turns the tile's
//     per-expert counts into its exclusive prefix.  Pass 2 replays the
//     match-any ranking to give every slot its rank among earlier slots of
//     the same expert.  The last CTA to finish turns the final inclusive
//     prefix into expert_count / expert_start and re-zeroes the scratch.
//
//  2. pack_rows_kernel  (the HBM-bound copy)
//     One warp per token: the token row is read ONCE into registers with
//     16-byte loads and stored to its K packed rows, pos = expert_start[e] +
//     rank.  It is launched as a programmatic dependent of kernel 1: its CTAs
//     start loading rows while kernel 1 is still scanning and only wait for
//     kernel 1 before reading rank / expert_start.
//
// The reference strategies replaced here re-read each token row once per slot
// (src/scatter/scatter_csort.cu:57-91, scatter_vec.cu:79-103) and pay a CUB
// sort or scan plus host-synchronising timers between launches.
#include <cuda_runtime.h>

#include "common.cuh"

namespace moe_b200 {

constexpr uint64_t kFlagAggregate = uint64_t(1) << 32;
constexpr uint64_t kFlagInclusive = uint64_t(2) << 32;

__device__ __forceinline__ void record_status(WsHeader* hdr, uint32_t bits) {
    atomicOr(&hdr->status, bits);
}

// Wait (bounded) until a look-back word is published; returns the word, or a
// zero aggregate after recording a timeout.
__device__ __forceinline__ uint64_t wait_status(const uint64_t* word, WsHeader* hdr) {
    uint64_t s = ld_relaxed_u64(word);
    uint32_t polls = 0;
    while ((s >> 32) == 0) {
        if (++polls > kMaxPolls) {
            record_status(hdr, MOE_B200_DEV_WAIT_TIMEOUT);
            return kFlagAggregate;
        }
        __nanosleep(64);
        s = ld_relaxed_u64(word);
    }
    return s;
}

// Loads the expert of slot idx for this lane; -1 for padding past T*K or for
// an out-of-range assignment (which is also recorded).
__device__ __forceinline__ int load_expert(const int32_t* __restrict__ asgn, int64_t idx,
                                           int64_t TK, int E, WsHeader* hdr) {
    if (idx >= TK) return -1;
    int e = __ldg(asgn + idx);
    if (e < 0 || e >= E) {
        record_status(hdr, MOE_B200_DEV_BAD_ASSIGNMENT);
        return -1;
    }
    return e;
}

__global__ void __launch_bounds__(kScanThreads)
route_scan_kernel(const int32_t* __restrict__ asgn, int64_t TK, int E, int tile_slots,
                  int num_tiles, WsHeader* __restrict__ hdr, uint64_t* __restrict__ status,
                  int32_t* __restrict__ rank, int32_t* __restrict__ expert_count,
                  int32_t* __restrict__ expert_start) {
    // Let the row-copy kernel get resident while this one scans.
    pdl_launch_dependents();

    extern __shared__ int32_t smem[];
    int32_t* hist = smem;                   // [kScanWarps][E]
    int32_t* tile_excl = smem + kScanWarps * E;  // [E] exclusive prefix of this tile
    int32_t* tile_agg = tile_excl + E;      // [E] this tile's counts
    __shared__ int s_tile;
    __shared__ int s_last;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) s_tile = int(atomicAdd(&hdr->ticket, 1u));
    for (int i = tid; i < kScanWarps * E; i += kScanThreads) hist[i] = 0;
    __syncthreads();
    const int tile = s_tile;

    // Each warp owns a contiguous run of the tile's slots.
    const int warp_slots = tile_slots / kScanWarps;
    const int64_t warp_base = int64_t(tile) * tile_slots + int64_t(warp) * warp_slots;
    int32_t* my_hist = hist + warp * E;
    const uint32_t lt = lanemask_lt();

    // Pass 1: per-warp histogram via match-any groups (one smem update per
    // distinct expert per 32 slots).
    for (int c = 0; c < warp_slots; c += kSlotsPerWarpChunk) {
        int e = load_expert(asgn, warp_base + c + lane, TK, E, hdr);
        uint32_t peers = __match_any_sync(0xffffffffu, e);
        if (e >= 0 && (peers & lt) == 0) my_hist[e] += __popc(peers);
        __syncwarp();
    }
    __syncthreads();

    // Per expert: exclusive prefix over the tile's warps; publish the tile
    // aggregate (tile 0 publishes its inclusive prefix directly).
    for (int e = tid; e < E; e += kScanThreads) {
        int32_t run = 0;
        for (int w = 0; w < kScanWarps; ++w) {
            int32_t v = hist[w * E + e];
            hist[w * E + e] = run;
            run += v;
        }
        tile_agg[e] = run;
        uint64_t flag = tile == 0 ? kFlagInclusive : kFlagAggregate;
        st_relaxed_u64(status + size_t(tile) * E + e, flag | uint32_t(run));
    }

    // Decoupled look-back, one thread per expert: walk predecessor tiles
    // (loads issued 8 at a time), summing aggregates until an inclusive prefix.
    for (int e = tid; e < E; e += kScanThreads) {
        int32_t excl = 0;
        if (tile > 0) {
            int j = tile - 1;
            bool found = false;
            while (!found && j >= 0) {
                uint64_t s[8];
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    s[i] = (j - i >= 0) ? ld_relaxed_u64(status + size_t(j - i) * E + e)
                                        : kFlagInclusive;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    if (found) break;
                    if (j - i < 0) { found = true; break; }
                    uint64_t w = s[i];
                    if ((w >> 32) == 0) w = wait_status(status + size_t(j - i) * E + e, hdr);
                    excl += int32_t(uint32_t(w));
                    if ((w >> 32) == 2) found = true;
                }
                j -= 8;
            }
        }
        tile_excl[e] = excl;
        st_relaxed_u64(status + size_t(tile) * E + e,
                       kFlagInclusive | uint32_t(excl + tile_agg[e]));
        // Seed every warp's running rank with the tile prefix.
        for (int w = 0; w < kScanWarps; ++w) hist[w * E + e] += excl;
    }
    __syncthreads();

    // Pass 2: replay the match-any ranking; rank = running count of the
    // expert before this slot (global across tiles).
    for (int c = 0; c < warp_slots; c += kSlotsPerWarpChunk) {
        int64_t idx = warp_base + c + lane;
        int e = (idx < TK) ? __ldg(asgn + idx) : -1;
        if (e >= E) e = -1;
        uint32_t peers = __match_any_sync(0xffffffffu, e);
        int32_t base = e >= 0 ? my_hist[e] : 0;
        __syncwarp();
        if (e >= 0 && (peers & lt) == 0) my_hist[e] = base + __popc(peers);
        __syncwarp();
        if (idx < TK) rank[idx] = e >= 0 ? base + __popc(peers & lt) : -1;
    }

    // The last CTA to finish publishes counts / starts and re-zeroes scratch.
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = (atomicAdd(&hdr->done, 1u) == uint32_t(num_tiles - 1));
    __syncthreads();
    if (!s_last) return;
    __threadfence();

    // Block-wide exclusive scan over E of the final inclusive counts: each
    // thread owns a contiguous run of experts.
    const int per = (E + kScanThreads - 1) / kScanThreads;
    const int e0 = tid * per;
    int32_t local = 0;
    for (int i = 0; i < per && e0 + i < E; ++i) {
        uint64_t w = ld_relaxed_u64(status + size_t(num_tiles - 1) * E + e0 + i);
        int32_t cnt = int32_t(uint32_t(w));
        tile_agg[e0 + i] = cnt;
        local += cnt;
    }
    // warp scan of thread totals, then across the 8 warps
    int32_t incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int32_t n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
    }
    __shared__ int32_t warp_tot[kScanWarps];
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    int32_t warp_off = 0;
    for (int w = 0; w < warp; ++w) warp_off += warp_tot[w];
    int32_t run = warp_off + incl - local;
    for (int i = 0; i < per && e0 + i < E; ++i) {
        int32_t cnt = tile_agg[e0 + i];
        expert_count[e0 + i] = cnt;
        expert_start[e0 + i] = run;
        run += cnt;
    }
    if (tid == kScanThreads - 1) expert_start[E] = warp_off + incl;

    // Leave the scratch zero-filled for the next call.
    const size_t words = size_t(num_tiles) * E;
    for (size_t i = tid; i < words; i += kScanThreads) status[i] = 0;
    if (tid == 0) {
        hdr->ticket = 0;
        hdr->done = 0;
    }
}

// One warp per token; VPL 16-byte vectors per lane per pass over the row.
template <int VPL>
__global__ void __launch_bounds__(256)
pack_rows_kernel(const uint4* __restrict__ emb, const int32_t* __restrict__ asgn,
                 const float* __restrict__ wts, const int32_t* __restrict__ rank,
                 const int32_t* __restrict__ expert_start, int T, int K, int nvec,
                 uint4* __restrict__ packed, float* __restrict__ packed_w,
                 int32_t* __restrict__ perm, int32_t* __restrict__ slot_pos) {
    const int lane = threadIdx.x & 31;
    const int warps_per_cta = blockDim.x >> 5;
    const int64_t gw = int64_t(blockIdx.x) * warps_per_cta + (threadIdx.x >> 5);
    const int64_t nw = int64_t(gridDim.x) * warps_per_cta;
    bool waited = false;

    for (int64_t t = gw; t < T; t += nw) {
        const uint4* src = emb + t * nvec;
        int e_lane = lane < K ? __ldg(asgn + t * K + lane) : 0;
        int32_t pos_lane = -1;
        for (int c0 = 0; c0 < nvec; c0 += 32 * VPL) {
            const bool full = c0 + 32 * VPL <= nvec;
            uint4 v[VPL];
            if (full) {
#pragma unroll
                for (int j = 0; j < VPL; ++j) v[j] = ld_nc_v4(src + c0 + j * 32 + lane);
            } else {
#pragma unroll
                for (int j = 0; j < VPL; ++j) {
                    int i = c0 + j * 32 + lane;
                    v[j] = i < nvec ? ld_nc_v4(src + i) : make_uint4(0, 0, 0, 0);
                }
            }
            if (c0 == 0) {
                if (!waited) {
                    pdl_wait_primary();
                    waited = true;
                }
                if (lane < K) {
                    int64_t s = t * K + lane;
                    int32_t r = rank[s];
                    if (r >= 0) {
                        pos_lane = __ldg(expert_start + e_lane) + r;
                        perm[pos_lane] = int32_t(t);
                        if (packed_w) packed_w[pos_lane] = __ldg(wts + s);
                    }
                    if (slot_pos) slot_pos[s] = pos_lane;
                }
            }
            for (int k = 0; k < K; ++k) {
                int32_t p = __shfl_sync(0xffffffffu, pos_lane, k);
                if (p < 0) continue;
                uint4* dst = packed + int64_t(p) * nvec + c0 + lane;
                if (full) {
#pragma unroll
                    for (int j = 0; j < VPL; ++j) st_v4(dst + j * 32, v[j]);
                } else {
#pragma unroll
                    for (int j = 0; j < VPL; ++j)
                        if (c0 + j * 32 + lane < nvec) st_v4(dst + j * 32, v[j]);
                }
            }
        }
    }
    if (!waited) pdl_wait_primary();
}

// Fallback for rows that are not 16-byte multiples / not 16-byte aligned:
// 2-byte elements, one warp per token.
__global__ void __launch_bounds__(256)
pack_rows_scalar_kernel(const uint16_t* __restrict__ emb, const int32_t* __restrict__ asgn,
                        const float* __restrict__ wts, const int32_t* __restrict__ rank,
                        const int32_t* __restrict__ expert_start, int T, int K, int d,
                        uint16_t* __restrict__ packed, float* __restrict__ packed_w,
                        int32_t* __restrict__ perm, int32_t* __restrict__ slot_pos) {
    pdl_wait_primary();
    const int lane = threadIdx.x & 31;
    const int warps_per_cta = blockDim.x >> 5;
    const int64_t gw = int64_t(blockIdx.x) * warps_per_cta + (threadIdx.x >> 5);
    const int64_t nw = int64_t(gridDim.x) * warps_per_cta;
    for (int64_t t = gw; t < T; t += nw) {
        int32_t pos_lane = -1;
        if (lane < K) {
            int64_t s = t * K + lane;
            int32_t r = rank[s];
            if (r >= 0) {
                pos_lane = __ldg(expert_start + __ldg(asgn + s)) + r;
                perm[pos_lane] = int32_t(t);
                if (packed_w) packed_w[pos_lane] = __ldg(wts + s);
            }
            if (slot_pos) slot_pos[s] = pos_lane;
        }
        for (int k = 0; k < K; ++k) {
            int32_t p = __shfl_sync(0xffffffffu, pos_lane, k);
            if (p < 0) continue;
            for (int i = lane; i < d; i += 32) packed[int64_t(p) * d + i] = emb[t * d + i];
        }
    }
}

// ----------------------------------------------------------------- host ----

static int sm_count() {
    int dev = 0, n = 148;
    if (cudaGetDevice(&dev) == cudaSuccess)
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n > 0 ? n : 148;
}

cudaError_t launch_pack(const void* emb, const int32_t* asgn, const float* wts, int T, int K,
                        int E, int d, void* packed, float* packed_w, int32_t* perm,
                        int32_t* expert_count, int32_t* expert_start, int32_t* slot_pos,
                        void* ws, cudaStream_t stream) {
    const PackPlan plan = plan_pack(T, K, E);
    char* base = static_cast<char*>(ws);
    WsHeader* hdr = reinterpret_cast<WsHeader*>(base);
    uint64_t* status = reinterpret_cast<uint64_t*>(base + plan.status_off);
    int32_t* rank = reinterpret_cast<int32_t*>(base + plan.rank_off);
    const int64_t TK = int64_t(T) * K;

    size_t smem = size_t(kScanWarps + 2) * E * sizeof(int32_t);
    route_scan_kernel<<<plan.num_tiles, kScanThreads, smem, stream>>>(
        asgn, TK, E, plan.tile_slots, plan.num_tiles, hdr, status, rank, expert_count,
        expert_start);
    cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) return err;

    const bool vec = (d % 8 == 0) && (reinterpret_cast<uintptr_t>(emb) % 16 == 0) &&
                     (reinterpret_cast<uintptr_t>(packed) % 16 == 0);
    const int threads = 256;
    const int warps_per_cta = threads / 32;
    int64_t want = (int64_t(T) + warps_per_cta - 1) / warps_per_cta;
    int64_t cap = int64_t(sm_count()) * 64;  // grid-stride beyond this
    int grid = int(want < cap ? want : cap);
    if (grid < 1) grid = 1;

    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (vec) {
        err = cudaLaunchKernelEx(&cfg, pack_rows_kernel<8>, static_cast<const uint4*>(emb), asgn,
                                 wts, static_cast<const int32_t*>(rank),
                                 static_cast<const int32_t*>(expert_start), T, K, d / 8,
                                 static_cast<uint4*>(packed), packed_w, perm, slot_pos);
    } else {
        err = cudaLaunchKernelEx(&cfg, pack_rows_scalar_kernel,
                                 static_cast<const uint16_t*>(emb), asgn, wts,
                                 static_cast<const int32_t*>(rank),
                                 static_cast<const int32_t*>(expert_start), T, K, d,
                                 static_cast<uint16_t*>(packed), packed_w, perm, slot_pos);
    }
    return err;
}

}  // namespace moe_b200
