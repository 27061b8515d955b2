// pack.cu -- stable MoE token packing for sm_100a.
//
// Output contract: moe::cpu_scatter (reference src/common/cpu_reference.cpp:
// 12-51): rows grouped by expert, ascending (t, k) inside each expert,
// perm / packed_weights / expert_count / expert_start bit-identical.
//
// Two kernels, one stream, no CUB and no host round trip:
//
//  1. route_scan_kernel  (reads T*K*4 bytes of assignments)
//     One CTA per tile of 2048 slots, tiles claimed in order through an
//     atomic ticket so that every earlier tile is already running (forward
//     progress of the look-back).  Per tile: each lane loads its 8 slots at
//     once; a warp-level __match_any_sync pass ranks every slot among the
//     earlier slots of the same expert in the warp and builds per-warp
//     histograms; a per-expert prefix over the warps and a decoupled look-back
//     across tiles (one thread per expert) turn that into a global rank.  The
//     last tile holds the final inclusive prefix and writes expert_count /
//     expert_start.
//
//  2. pack_rows_kernel  (the HBM-bound copy)
//     One warp per token: the token row is read ONCE into registers with
//     16-byte loads and stored to its K packed rows, pos = expert_start[e] +
//     rank.  It is launched as a programmatic dependent of kernel 1: its CTAs
//     start loading rows while kernel 1 is still scanning and only wait for
//     kernel 1 before reading rank / expert_start; afterwards they re-zero the
//     look-back scratch for the next call.
//
// The reference strategies replaced here re-read each token row once per slot
// (src/scatter/scatter_csort.cu:57-91, scatter_vec.cu:79-103) and pay a CUB
// sort or scan plus host-synchronising timers between launches.
#include <algorithm>
#include <cstdlib>

#include <cuda_runtime.h>

#include "common.cuh"

namespace moe_b200 {

constexpr uint64_t kFlagAggregate = uint64_t(1) << 32;
constexpr uint64_t kFlagInclusive = uint64_t(2) << 32;
// Shared-memory row ring of the bulk packer (per CTA; two CTAs per SM).
constexpr size_t kPackRingBytes = 100 * 1024;

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

// Raw assignment of slot idx (-1 past the end).
__device__ __forceinline__ int load_slot(const int32_t* __restrict__ asgn, int64_t idx, int64_t TK) {
    return idx < TK ? __ldg(asgn + idx) : -1;
}

__global__ void __launch_bounds__(kScanThreads)
route_scan_kernel(const int32_t* __restrict__ asgn, int64_t TK, int E, int num_tiles,
                  WsHeader* __restrict__ hdr, uint64_t* __restrict__ status,
                  int32_t* __restrict__ rank, int32_t* __restrict__ expert_count,
                  int32_t* __restrict__ expert_start, EpPublish pub) {
    extern __shared__ int32_t smem[];
    int32_t* hist = smem;                        // [kScanWarps][E]
    int32_t* tile_excl = smem + kScanWarps * E;  // [E] exclusive prefix of this tile
    int32_t* tile_agg = tile_excl + E;           // [E] this tile's counts
    __shared__ int s_tile;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t lt = lanemask_lt();

    // Tiles are claimed through a ticket so that every earlier tile is already
    // running when this one looks back.  The slots of the likely tile
    // (blockIdx.x) are loaded while the ticket round-trip is in flight.
    int tile = blockIdx.x;
    int e[kScanChunks];
    {
        const int64_t base = int64_t(tile) * kTileSlots + warp * (kScanChunks * 32) + lane;
#pragma unroll
        for (int c = 0; c < kScanChunks; ++c) e[c] = load_slot(asgn, base + c * 32, TK);
    }
    if (tid == 0) s_tile = int(atomicAdd(&hdr->ticket, 1u));
    for (int i = tid; i < kScanWarps * E; i += kScanThreads) hist[i] = 0;
    __syncthreads();
    if (s_tile != tile) {  // CTA-uniform; rare
        tile = s_tile;
        const int64_t base = int64_t(tile) * kTileSlots + warp * (kScanChunks * 32) + lane;
#pragma unroll
        for (int c = 0; c < kScanChunks; ++c) e[c] = load_slot(asgn, base + c * 32, TK);
    }
    const int64_t warp_base = int64_t(tile) * kTileSlots + warp * (kScanChunks * 32);

    // Per-warp ranking via match-any groups, in slot order: r = earlier slots
    // of the same expert within this warp's run; one smem update per group.
    int32_t* my_hist = hist + warp * E;
    int r[kScanChunks];
#pragma unroll
    for (int c = 0; c < kScanChunks; ++c) {
        int ec = e[c];
        if (ec >= E || (ec < 0 && warp_base + c * 32 + lane < TK)) {
            record_status(hdr, MOE_B200_DEV_BAD_ASSIGNMENT);
            ec = -1;
        }
        e[c] = ec;
        const uint32_t peers = __match_any_sync(0xffffffffu, ec);
        const int32_t b = ec >= 0 ? my_hist[ec] : 0;
        __syncwarp();
        if (ec >= 0 && (peers & lt) == 0) my_hist[ec] = b + __popc(peers);
        __syncwarp();
        r[c] = b + __popc(peers & lt);
    }
    __syncthreads();
    // The assignments are in registers: let the row-copy kernel start its
    // row prefetch now (its loads would otherwise queue ahead of ours).
    pdl_launch_dependents();

    // Per expert: exclusive prefix over the tile's warps; publish the tile
    // aggregate (tile 0 publishes its inclusive prefix directly).
    for (int x = tid; x < E; x += kScanThreads) {
        int32_t run = 0;
#pragma unroll
        for (int w = 0; w < kScanWarps; ++w) {
            int32_t v = hist[w * E + x];
            hist[w * E + x] = run;
            run += v;
        }
        tile_agg[x] = run;
        st_relaxed_u64(status + size_t(tile) * E + x,
                       (tile == 0 ? kFlagInclusive : kFlagAggregate) | uint32_t(run));
    }

    // Decoupled look-back, one thread per expert: predecessor words are loaded
    // kWindow at a time; aggregates are summed until an inclusive prefix.
    constexpr int kWindow = 8;
    for (int x = tid; x < E; x += kScanThreads) {
        int32_t excl = 0;
        int j = tile - 1;
        bool found = tile == 0;
        while (!found) {
            uint64_t w8[kWindow];
#pragma unroll
            for (int i = 0; i < kWindow; ++i)
                w8[i] = (j - i >= 0) ? ld_relaxed_u64(status + size_t(j - i) * E + x) : kFlagInclusive;
#pragma unroll
            for (int i = 0; i < kWindow; ++i) {
                if (!found) {
                    uint64_t w = w8[i];
                    if (j - i >= 0 && (w >> 32) == 0) w = wait_status(status + size_t(j - i) * E + x, hdr);
                    excl += int32_t(uint32_t(w));
                    if ((w >> 32) == 2) found = true;
                }
            }
            j -= kWindow;
        }
        tile_excl[x] = excl;
        if (tile > 0)
            st_relaxed_u64(status + size_t(tile) * E + x, kFlagInclusive | uint32_t(excl + tile_agg[x]));
    }
    __syncthreads();

#pragma unroll
    for (int c = 0; c < kScanChunks; ++c) {
        const int64_t idx = warp_base + c * 32 + lane;
        if (idx < TK) rank[idx] = e[c] >= 0 ? tile_excl[e[c]] + my_hist[e[c]] + r[c] : -1;
    }

    // The last tile holds the final inclusive prefix: publish counts / starts.
    if (tile != num_tiles - 1) return;
    const int per = (E + kScanThreads - 1) / kScanThreads;
    const int e0 = tid * per;
    int32_t local = 0;
    for (int i = 0; i < per && e0 + i < E; ++i) local += tile_excl[e0 + i] + tile_agg[e0 + i];
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
        const int32_t cnt = tile_excl[e0 + i] + tile_agg[e0 + i];
        expert_count[e0 + i] = cnt;
        expert_start[e0 + i] = run;
        run += cnt;
        // expert parallel: the counts go straight into every rank's inbox
        for (int p = 0; pub.peer && p < pub.nranks; ++p)
            reinterpret_cast<int32_t*>(pub.peer[p] + pub.off_inbox)[size_t(pub.rank) * E + e0 + i] = cnt;
    }
    if (tid == kScanThreads - 1) expert_start[E] = warp_off + incl;
    if (pub.peer) {
        __threadfence_system();
        __syncthreads();
        if (tid < pub.nranks)
            st_release_sys(reinterpret_cast<uint64_t*>(pub.peer[tid] + pub.off_flag) + pub.rank, pub.epoch);
    }
}


// One warp per token; VPL 16-byte vectors per lane per pass over the row.
template <int VPL>
__global__ void __launch_bounds__(256)
pack_rows_kernel(const uint4* __restrict__ emb, const int32_t* __restrict__ asgn,
                 const float* __restrict__ wts, const int32_t* __restrict__ rank,
                 const int32_t* __restrict__ expert_start, int T, int K, int nvec,
                 uint4* __restrict__ packed, float* __restrict__ packed_w,
                 int32_t* __restrict__ perm, int32_t* __restrict__ slot_pos,
                 WsHeader* __restrict__ hdr, uint64_t* __restrict__ status, size_t status_words) {
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
    rearm_scan_scratch(hdr, status, status_words);
}

// Persistent TMA bulk-copy row packer: one warp per CTA, a ring of R row
// slots in shared memory.  Each CTA owns a contiguous token range.  Before
// its PDL wait it issues cp.async.bulk loads of its first R token rows (the
// rows are kernel inputs, so this overlaps the route/scan kernel).  After the
// wait it computes the K packed positions of a group of G = 32 / K tokens at
// once (lane l -> slot l % K of token l / K; expert_start cached in shared
// memory), stores every row with K cp.async.bulk shared->global copies, and
// refills a slot with the row R tokens ahead once the stores of the row it
// held (issued kLag tokens earlier) have finished reading it.
constexpr int kBulkLag = 2;

__global__ void __launch_bounds__(32)
pack_rows_bulk_kernel(const uint16_t* __restrict__ emb, const int32_t* __restrict__ asgn,
                      const float* __restrict__ wts, const int32_t* __restrict__ rank,
                      const int32_t* __restrict__ expert_start, int T, int K, int E, int d,
                      int ring, uint16_t* __restrict__ packed, float* __restrict__ packed_w,
                      int32_t* __restrict__ perm, int32_t* __restrict__ slot_pos,
                      WsHeader* __restrict__ hdr, uint64_t* __restrict__ status,
                      size_t status_words) {
    extern __shared__ __align__(128) unsigned char ring_smem[];
    const uint32_t rowb = uint32_t(d) * 2;
    uint64_t* full = reinterpret_cast<uint64_t*>(ring_smem + size_t(ring) * rowb);
    int32_t* s_start = reinterpret_cast<int32_t*>(full + ring);  // [E]
    const int lane = threadIdx.x;

    const int64_t per = (int64_t(T) + gridDim.x - 1) / gridDim.x;
    const int64_t t0 = int64_t(blockIdx.x) * per;
    const int64_t n = t0 < T ? (T - t0 < per ? T - t0 : per) : 0;

    if (lane == 0) {
        for (int r = 0; r < ring; ++r) mbar_init(full + r, 1);
        mbar_fence_init();
    }
    __syncwarp();
    // Prefetch the first rows: inputs only, so no need to wait for the scan.
    const int64_t pre = n < ring ? n : ring;
    int64_t issued = pre;  // rows 0 .. issued-1 have had their load issued (in order)
    if (lane == 0) {
        for (int64_t i = 0; i < pre; ++i) {
            mbar_arrive_expect_tx(full + i, rowb);
            bulk_g2s(ring_smem + size_t(i) * rowb, emb + (t0 + i) * d, rowb, full + i);
        }
    }
    const int G = 32 / K;
    const int gk = lane % K, gi = lane / K;
    const bool lane_used = gi < G;
    // Group inputs that do not depend on the scan.
    auto load_inputs = [&](int64_t g, int& e, float& w) {
        const int64_t i = g * G + gi;
        e = -1;
        w = 0.f;
        if (lane_used && i < n) {
            const int64_t s = (t0 + i) * K + gk;
            e = __ldg(asgn + s);
            if (packed_w) w = __ldg(wts + s);
        }
    };
    int e_cur, e_nxt;
    float w_cur, w_nxt;
    load_inputs(0, e_cur, w_cur);

    pdl_wait_primary();
    rearm_scan_scratch(hdr, status, status_words);
    for (int x = lane; x < E; x += 32) s_start[x] = expert_start[x];
    __syncwarp();

    // Position of this lane's slot in group g (after the scan).
    auto position = [&](int64_t g, int e) -> int32_t {
        const int64_t i = g * G + gi;
        if (!lane_used || i >= n) return -1;
        const int64_t s = (t0 + i) * K + gk;
        const int32_t r = rank[s];
        const int32_t pos = (r >= 0 && e >= 0 && e < E) ? s_start[e] + r : -1;
        if (slot_pos) slot_pos[s] = pos;
        return pos;
    };
    int32_t p_cur = position(0, e_cur);

    bool ok = true;
    for (int64_t g = 0; ok && g * G < n; ++g) {
        load_inputs(g + 1, e_nxt, w_nxt);
        if (p_cur >= 0) {
            perm[p_cur] = int32_t(t0 + g * G + gi);
            if (packed_w) packed_w[p_cur] = w_cur;
        }
        for (int q = 0; q < G; ++q) {
            const int64_t i = g * G + q;
            if (i >= n) break;
            const int slot = int(i % ring);
            if (!mbar_wait(full + slot, uint32_t(i / ring) & 1u)) {
                if (lane == 0) atomicOr(&hdr->status, MOE_B200_DEV_WAIT_TIMEOUT);
                ok = false;
                break;
            }
            if (lane_used && gi == q && p_cur >= 0)
                bulk_s2g(packed + int64_t(p_cur) * d, ring_smem + size_t(slot) * rowb, rowb);
            bulk_commit();
            // Refill the slot of token i - kLag once its stores have read it.
            const int64_t j = i - kBulkLag;
            if (j >= 0 && j + ring < n) {
                bulk_wait_read<kBulkLag>();
                __syncwarp();
                if (lane == 0) {
                    const int js = int(j % ring);
                    mbar_arrive_expect_tx(full + js, rowb);
                    bulk_g2s(ring_smem + size_t(js) * rowb, emb + (t0 + j + ring) * d, rowb, full + js);
                }
                issued = j + ring + 1;
            }
        }
        e_cur = e_nxt;
        w_cur = w_nxt;
        if (ok) p_cur = position(g + 1, e_cur);
    }
    // Every store must finish before the shared memory it reads goes away,
    // and (after an abort) every row load still in flight must have landed.
    bulk_wait<0>();
    if (!ok && lane == 0) drain_stages(full, uint32_t(issued), ring);  // normally every load was waited for
    __syncwarp();
    pdl_launch_dependents();
}

// Indices only (packed == NULL): perm / packed_weights / slot_pos from the
// scan, no row copy -- for consumers that gather the rows themselves
// (moe_b200_grouped_swiglu_gather).  Thread per slot.
__global__ void __launch_bounds__(256)
pack_index_kernel(const int32_t* __restrict__ asgn, const float* __restrict__ wts,
                  const int32_t* __restrict__ rank, const int32_t* __restrict__ expert_start, int64_t TK, int K,
                  int E, float* __restrict__ packed_w, int32_t* __restrict__ perm, int32_t* __restrict__ slot_pos,
                  WsHeader* __restrict__ hdr, uint64_t* __restrict__ status, size_t status_words) {
    pdl_wait_primary();
    rearm_scan_scratch(hdr, status, status_words);
    const int64_t nt = int64_t(gridDim.x) * blockDim.x;
    for (int64_t s = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; s < TK; s += nt) {
        const int32_t r = rank[s];
        const int e = __ldg(asgn + s);
        int32_t pos = -1;
        if (r >= 0 && e >= 0 && e < E) {
            pos = expert_start[e] + r;
            perm[pos] = int32_t(s / K);
            if (packed_w) packed_w[pos] = __ldg(wts + s);
        }
        if (slot_pos) slot_pos[s] = pos;
    }
    pdl_launch_dependents();
}

// Fallback for rows that are not 16-byte multiples / not 16-byte aligned:
// 2-byte elements, one warp per token.
__global__ void __launch_bounds__(256)
pack_rows_scalar_kernel(const uint16_t* __restrict__ emb, const int32_t* __restrict__ asgn,
                        const float* __restrict__ wts, const int32_t* __restrict__ rank,
                        const int32_t* __restrict__ expert_start, int T, int K, int d,
                        uint16_t* __restrict__ packed, float* __restrict__ packed_w,
                        int32_t* __restrict__ perm, int32_t* __restrict__ slot_pos,
                        WsHeader* __restrict__ hdr, uint64_t* __restrict__ status,
                        size_t status_words) {
    pdl_wait_primary();
    rearm_scan_scratch(hdr, status, status_words);
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

// Enqueues the route/scan kernel alone (ranks in the workspace, counts and
// starts in the outputs); used by launch_pack and by the expert-parallel
// dispatch.
cudaError_t launch_route_scan(const int32_t* asgn, int T, int K, int E, int32_t* expert_count,
                              int32_t* expert_start, void* ws, cudaStream_t stream, const EpPublish* pub) {
    const PackPlan plan = plan_pack(T, K, E);
    char* base = static_cast<char*>(ws);
    size_t smem = size_t(kScanWarps + 2) * E * sizeof(int32_t);
    EpPublish none{};
    route_scan_kernel<<<plan.num_tiles, kScanThreads, smem, stream>>>(
        asgn, int64_t(T) * K, E, plan.num_tiles, reinterpret_cast<WsHeader*>(base),
        reinterpret_cast<uint64_t*>(base + plan.status_off),
        reinterpret_cast<int32_t*>(base + plan.rank_off), expert_count, expert_start, pub ? *pub : none);
    return cudaGetLastError();
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
    const size_t words = size_t(plan.num_tiles) * size_t(E);

    cudaError_t err = launch_route_scan(asgn, T, K, E, expert_count, expert_start, ws, stream, nullptr);
    if (err != cudaSuccess) return err;
    if (!packed) {
        cudaLaunchConfig_t cfg = pdl_config(dim3(unsigned(std::min<int64_t>((TK + 255) / 256, int64_t(sm_count()) * 8))),
                                            dim3(256), 0, stream);
        cudaLaunchAttribute attr = pdl_attr();
        cfg.attrs = &attr;
        cfg.numAttrs = 1;
        return cudaLaunchKernelEx(&cfg, pack_index_kernel, asgn, wts, static_cast<const int32_t*>(rank),
                                  static_cast<const int32_t*>(expert_start), TK, K, E, packed_w, perm, slot_pos,
                                  hdr, status, words);
    }

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
    const size_t rowb = size_t(d) * 2;
    const int ring = int(kPackRingBytes / rowb) < 64 ? int(kPackRingBytes / rowb) : 64;
    const char* sel = getenv("MOE_B200_PACK");
    const bool want_bulk = !(sel && sel[0] == 'r');
    if (vec && want_bulk && ring >= 4) {
        const int smem = int(ring * rowb + ring * 8 + E * 4 + 128);
        err = cudaFuncSetAttribute(pack_rows_bulk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   smem);
        if (err != cudaSuccess) return err;
        int per_sm = 0;
        err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, pack_rows_bulk_kernel, 32, smem);
        if (err != cudaSuccess) return err;
        if (per_sm < 1) per_sm = 1;
        int64_t g = int64_t(sm_count()) * per_sm;
        // keep at least a few tokens per CTA so the ring is used
        int64_t gmax = (int64_t(T) + 3) / 4;
        if (g > gmax) g = gmax;
        if (g < 1) g = 1;
        cfg.gridDim = dim3(unsigned(g));
        cfg.blockDim = dim3(32);
        cfg.dynamicSmemBytes = size_t(smem);
        err = cudaLaunchKernelEx(&cfg, pack_rows_bulk_kernel, static_cast<const uint16_t*>(emb), asgn,
                                 wts, static_cast<const int32_t*>(rank),
                                 static_cast<const int32_t*>(expert_start), T, K, E, d, ring,
                                 static_cast<uint16_t*>(packed), packed_w, perm, slot_pos, hdr, status,
                                 words);
    } else if (vec) {
        err = cudaLaunchKernelEx(&cfg, pack_rows_kernel<8>, static_cast<const uint4*>(emb), asgn,
                                 wts, static_cast<const int32_t*>(rank),
                                 static_cast<const int32_t*>(expert_start), T, K, d / 8,
                                 static_cast<uint4*>(packed), packed_w, perm, slot_pos, hdr,
                                 status, words);
    } else {
        err = cudaLaunchKernelEx(&cfg, pack_rows_scalar_kernel,
                                 static_cast<const uint16_t*>(emb), asgn, wts,
                                 static_cast<const int32_t*>(rank),
                                 static_cast<const int32_t*>(expert_start), T, K, d,
                                 static_cast<uint16_t*>(packed), packed_w, perm, slot_pos, hdr,
                                 status, words);
    }
    return err;
}

}  // namespace moe_b200
