// ep_p2p.cu -- fused expert-parallel dispatch and combine over peer memory
// (NVLink / NVSwitch), one process per GPU.
//
// Each rank owns one symmetric region (one cudaMalloc, the same layout on
// every rank) that its peers map through CUDA IPC:
//   [counts flags | data flags | back flags]  one u64 epoch word per sender
//   inbox  [N][E] int32        every rank's expert counts for this step
//   recv   [N * max_tokens * K][d]   rows routed to this rank's experts,
//                              expert-major (see below)
//   ret    [N * max_tokens * K] int64  return address of every received row:
//                              sender << 32 | the sender's packed row
//   back   [max_tokens * K][d] this rank's rows after their expert, in its
//                              own packed order
// One step (epoch e, the same on all ranks; epochs only grow, so no flag is
// ever reset), on one stream: four launches for the identity expert, six for
// the SwiGLU expert:
//   1. route_scan (pack.cu): local counts / starts / ranks; the tile that
//      finishes the scan writes the counts into every peer's inbox and raises
//      counts flag = e on every peer (system-scope release)
//   2. ep_pack_dispatch_kernel: wait for all counts, then every token row is
//      read once and stored K times straight into the receive buffer of the
//      rank owning each slot's expert (NVLink stores); the last CTA raises
//      data flag = e on every peer
//   3. ep_receive_kernel (receiver; the SwiGLU expert only): the segment
//      table of the receive buffer.  Called alone (moe_b200_ep_receive) it
//      first waits for all data flags, so any expert kernel may follow; in
//      the one-call step it waits for the counts only and the gate/up GEMM
//      waits for the data flags itself, after the replicated experts' rows
//   4. the expert: grouped SwiGLU whose down-GEMM epilogue stores every row
//      straight into the sender's back buffer (grouped_ffn.cu scatter mode),
//      or ep_return_identity_kernel (which waits for the data flags itself);
//      the last CTA of either raises back flag = e on every peer
//   5. unpermute (unpermute.cu): its copy warps wait for all back flags, then
//      combine the local back buffer
// Replicated ("hot") experts: every rank holds its own copy of the experts in
// a set H (the same on all ranks, moe_b200_ep_set_replicated); a row routed
// to an expert of H never leaves its rank.  Receive buffer of rank r,
// expert-major so that every local expert is ONE contiguous segment for the
// grouped FFN (sender-major (sender, expert) pieces of a few dozen rows each
// would waste most of every 128-row tile at 8 ranks):
//   [r's 1st non-replicated expert: rows of sender 0, sender 1, ..., N-1]
//   [r's 2nd non-replicated expert: ...] ... [own rows of the replicated
//   experts, expert-major]
// and r's local expert weights are ordered [non-replicated experts of its
// range, ascending] + [replicated experts, ascending].  Each received row's
// return address travels with it (the dispatch stores it into `ret`), so the
// return needs no per-sender table.
// The host never waits inside a step.  This replaces the reference's
// AllGather -> D2H -> host offsets -> grouped ncclSend/ncclRecv exchange
// (apps/bench_prefill.cu:768-807, 889-906).  Every wait is bounded (the
// context's timeout); on expiry the kernel sets MOE_B200_DEV_WAIT_TIMEOUT in
// the library's device status word and carries on.  Only plain loads and
// stores touch peer memory (no TMA, no multicast).
#include <cstring>
#include <mutex>

#include <cuda_runtime.h>

#include "common.cuh"

namespace moe_b200 {

int fail(int code, const char* fmt, ...);
int cuda_fail(cudaError_t err, const char* where);
cudaError_t launch_route_scan(const int32_t* asgn, int T, int K, int E, int32_t* expert_count,
                              int32_t* expert_start, void* ws, cudaStream_t stream, const EpPublish* pub);
cudaError_t launch_unpermute(const void* y, const float* packed_w, const int32_t* slot_pos, int T, int K,
                             int d, int dtype, void* out, cudaStream_t stream, const EpWait* wait);
int grouped_swiglu_impl(const void* x, const int32_t* seg_start, const int32_t* seg_expert, int nseg, int rows,
                        int d, int I, int E, const void* w_gate_up, const void* w_down, int dtype, void* h,
                        void* y, cudaStream_t s, char* const* dst_base, const int64_t* row_ret,
                        const int32_t* gather_rows, int gather_T, const EpSignal* sig, const EpWait* rows_wait,
                        int wait_seg0);

constexpr int kEpMaxRanks = 64;

constexpr int kEpMaxExperts = 1024;
constexpr int kInboxSmemMax = 4096;  // counts copied to shared memory up to N*E of this (16 KB)

struct EpGeom {
    int nranks, rank, E, K, d, max_tokens;
    int first[kEpMaxRanks + 1];
    uint32_t hot[kEpMaxExperts / 32];  // replicated experts (bit e)
    int nhot;                          // |H|
    int lrange;                        // experts of this rank's range that are not replicated
    size_t off_cflag, off_dflag, off_bflag, off_count, off_inbox, off_recv, off_ret, off_back, total;
    int64_t recv_cap;
    uint64_t timeout_ns;
};

struct EpContext {
    EpGeom g;
    int device = -1;
    char* region = nullptr;
    char* peer_host[kEpMaxRanks] = {};
    bool opened[kEpMaxRanks] = {};
    char** peer_dev = nullptr;   // device array: every rank's region in this address space
    char** back_dev = nullptr;   // device array: every rank's back buffer
    bool connected = false;
    uint64_t epoch = 0;          // largest epoch enqueued so far
    int32_t* seg = nullptr;      // moe_b200_ep_step's segment table: [E + 1] starts + [E] experts
};

static size_t al4k(size_t x) { return (x + 4095) & ~size_t(4095); }

// ---------------------------------------------------------------- device ----

__host__ __device__ __forceinline__ bool ep_is_hot(const EpGeom& g, int e) {
    return (g.hot[e >> 5] >> (e & 31)) & 1u;
}

// Bounded wait until flags[i] >= epoch for i in [0, n), one thread per flag.
// Returns false (and records a timeout) if any flag did not arrive in time.
__device__ bool wait_flags(const uint64_t* flags, int n, uint64_t epoch, uint64_t timeout_ns,
                           uint32_t* dev_status, int* s_fail) {
    if (threadIdx.x < n) {
        const uint64_t t0 = globaltimer_ns();
        while (ld_acquire_sys(flags + threadIdx.x) < epoch) {
            if (globaltimer_ns() - t0 > timeout_ns) {
                atomicOr(dev_status, MOE_B200_DEV_WAIT_TIMEOUT);
                *s_fail = 1;
                break;
            }
            __nanosleep(100);
        }
    }
    __syncthreads();
    return *s_fail == 0;
}

// ld_nc_v4 as a volatile asm statement, so it keeps its place before the
// (volatile) row stores that follow it in program order.
__device__ __forceinline__ uint4 ld_nc_v4_first(const uint4* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

// Warp per token: row read once (16-byte loads), stored to the receive buffer
// of the rank owning each slot's expert.
__global__ void __launch_bounds__(256)
ep_pack_dispatch_kernel(EpGeom g, char* const* __restrict__ peer, const uint4* __restrict__ emb,
                        const int32_t* __restrict__ asgn, const float* __restrict__ wts,
                        const int32_t* __restrict__ rank, const int32_t* __restrict__ expert_start, int T,
                        float* __restrict__ packed_w, int32_t* __restrict__ perm,
                        int32_t* __restrict__ slot_pos, WsHeader* __restrict__ hdr,
                        uint64_t* __restrict__ status, size_t status_words, uint64_t epoch,
                        uint32_t* __restrict__ dev_status, int inbox_smem) {
    __shared__ int s_fail;
    // per expert e: the rank whose receive buffer takes its rows, and the
    // receive row of packed position p there = s_dst[e] + p
    extern __shared__ int64_t s_dst[];                          // [E]
    int32_t* s_owner = reinterpret_cast<int32_t*>(s_dst + g.E);  // [E]
    int32_t* s_start = s_owner + g.E;                            // [E] this rank's packed expert starts
    int32_t* s_inbox = s_start + g.E;                            // [N][E] when inbox_smem
    const int K = g.K, nvec = g.d / 8;
    if (threadIdx.x == 0) s_fail = 0;
    __syncthreads();
    pdl_wait_primary();
    rearm_scan_scratch(hdr, status, status_words);
    const char* mine = peer[g.rank];
    wait_flags(reinterpret_cast<const uint64_t*>(mine + g.off_cflag), g.nranks, epoch, g.timeout_ns, dev_status,
               &s_fail);
    const int32_t* inbox = reinterpret_cast<const int32_t*>(mine + g.off_inbox);
    // one coalesced pass over every rank's counts and this rank's starts, so
    // the serial offset loops below read shared memory instead of chains of
    // global loads while the rest of the CTA waits at the barrier
    for (int e = threadIdx.x; e < g.E; e += blockDim.x) s_start[e] = expert_start[e];
    if (inbox_smem) {
        for (int i = threadIdx.x; i < g.nranks * g.E; i += blockDim.x) s_inbox[i] = inbox[i];
        inbox = s_inbox;
    }
    __syncthreads();
    const int32_t* own = inbox + size_t(g.rank) * g.E;  // this rank's counts
    // Receiver r (thread r): its own rows of the replicated experts first
    // (written by its own dispatch, so its gate/up GEMM can start on them
    // before the other senders' rows land), then its non-replicated experts
    // in ascending order, each holding every sender's rows in sender order;
    // this sender's rows of expert e start after all senders' rows of r's
    // earlier experts and the rows of senders < rank of expert e.
    if (threadIdx.x < g.nranks) {
        const int r = threadIdx.x;
        int64_t base = 0;
        for (int e = 0; g.nhot > 0 && e < g.E; ++e)
            if (ep_is_hot(g, e)) base += inbox[r * g.E + e];
        for (int e = g.first[r]; e < g.first[r + 1]; ++e) {
            if (ep_is_hot(g, e)) continue;
            int64_t before = 0, col = 0;
            for (int s = 0; s < g.nranks; ++s) {
                const int32_t c = inbox[s * g.E + e];
                col += c;
                before += s < g.rank ? c : 0;
            }
            s_owner[e] = r;
            s_dst[e] = base + before - s_start[e];
            base += col;
        }
    } else if (threadIdx.x == g.nranks && g.nhot > 0) {
        // this rank's rows of the replicated experts: the head of its own
        // receive buffer
        int64_t base = 0;
        for (int e = 0; e < g.E; ++e) {
            if (!ep_is_hot(g, e)) continue;
            s_owner[e] = g.rank;
            s_dst[e] = base - s_start[e];
            base += own[e];
        }
    }
    __syncthreads();

    const int lane = threadIdx.x & 31;
    const int64_t gw = int64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int64_t nw = int64_t(gridDim.x) * (blockDim.x >> 5);
    const size_t rowb = size_t(g.d) * 2;
    constexpr int VPL = 8;
    for (int64_t t = gw; t < T && !s_fail; t += nw) {
        uint4* dst_lane = nullptr;
        if (lane < K) {
            const int64_t sidx = t * K + lane;
            const int32_t r = rank[sidx];
            int32_t p = -1;
            if (r >= 0) {
                const int e = __ldg(asgn + sidx);
                p = s_start[e] + r;
                perm[p] = int32_t(t);
                if (packed_w) packed_w[p] = __ldg(wts + sidx);
                const int owner = s_owner[e];
                const int64_t rrow = s_dst[e] + p;
                dst_lane = reinterpret_cast<uint4*>(peer[owner] + g.off_recv + size_t(rrow) * rowb);
                // the row's return address travels with it
                reinterpret_cast<int64_t*>(peer[owner] + g.off_ret)[rrow] =
                    (int64_t(g.rank) << 32) | int64_t(uint32_t(p));
            }
            if (slot_pos) slot_pos[sidx] = p;
        }
        const uint4* src = emb + t * nvec;
        for (int c0 = 0; c0 < nvec; c0 += 32 * VPL) {
            uint4 v[VPL];
#pragma unroll
            for (int j = 0; j < VPL; ++j) {
                const int i = c0 + j * 32 + lane;
                v[j] = i < nvec ? ld_nc_v4_first(src + i) : make_uint4(0, 0, 0, 0);
            }
            for (int k = 0; k < K; ++k) {
                uint4* dst = reinterpret_cast<uint4*>(__shfl_sync(0xffffffffu, reinterpret_cast<uintptr_t>(dst_lane), k));
                if (!dst) continue;
#pragma unroll
                for (int j = 0; j < VPL; ++j) {
                    const int i = c0 + j * 32 + lane;
                    if (i < nvec) st_v4(dst + i, v[j]);
                }
            }
        }
    }
    // The last CTA to finish announces the rows to every receiver (unless a
    // CTA gave up waiting for the counts: then the receivers time out too).
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0)
        ep_signal_done(EpSignal{peer, g.off_dflag, hdr->pad, g.rank, g.nranks, epoch}, s_fail != 0);
}

// Receiver: wait for every sender's rows (wait_rows) or only for its counts,
// then the segment table of the receive buffer: one segment per local
// expert, the own rows of the replicated experts first, then the range's
// non-replicated experts with every sender's rows; seg_expert = the local
// expert index (local experts are numbered non-replicated first, replicated
// last).  Counts only: the kernels that read the rows wait for the senders'
// data flags themselves.
__global__ void __launch_bounds__(256)
ep_receive_kernel(EpGeom g, char* const* __restrict__ peer, uint64_t epoch, int32_t* __restrict__ seg_start,
                  int32_t* __restrict__ seg_expert, uint32_t* __restrict__ dev_status, int inbox_smem,
                  int wait_rows) {
    extern __shared__ int32_t s_inbox[];  // [N][E] when inbox_smem
    __shared__ int s_fail;
    __shared__ int32_t warp_tot[8];
    __shared__ int32_t carry;
    if (threadIdx.x == 0) {
        s_fail = 0;
        carry = 0;
    }
    __syncthreads();
    const char* mine = peer[g.rank];
    wait_flags(reinterpret_cast<const uint64_t*>(mine + (wait_rows ? g.off_dflag : g.off_cflag)), g.nranks, epoch,
               g.timeout_ns, dev_status, &s_fail);
    const int32_t* inbox = reinterpret_cast<const int32_t*>(mine + g.off_inbox);
    if (inbox_smem) {
        for (int i = threadIdx.x; i < g.nranks * g.E; i += blockDim.x) s_inbox[i] = inbox[i];
        inbox = s_inbox;   // published by the __syncthreads below
    }
    // segments in buffer order: [replicated] + [non-replicated of the range]
    __shared__ int16_t s_local[kEpMaxExperts];
    if (threadIdx.x == 0) {
        int n = 0;
        for (int e = 0; e < g.E; ++e)
            if (ep_is_hot(g, e)) s_local[n++] = int16_t(e);
        for (int e = g.first[g.rank]; e < g.first[g.rank + 1]; ++e)
            if (!ep_is_hot(g, e)) s_local[n++] = int16_t(e);
    }
    __syncthreads();
    const int L = g.lrange, H = g.nhot;
    const int nseg = L + H;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int base = 0; base < nseg; base += blockDim.x) {
        const int j = base + tid;
        int32_t v = 0;
        if (j < nseg) {
            const int e = s_local[j];
            if (j < H) {
                v = inbox[g.rank * g.E + e];
                seg_expert[j] = L + j;
            } else {
                for (int s = 0; s < g.nranks; ++s) v += inbox[s * g.E + e];
                seg_expert[j] = j - H;
            }
        }
        int32_t incl = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int32_t n = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += n;
        }
        if (lane == 31) warp_tot[warp] = incl;
        __syncthreads();
        int32_t off = carry;
        for (int w = 0; w < warp; ++w) off += warp_tot[w];
        if (j < nseg) seg_start[j] = off + incl - v;
        __syncthreads();
        if (tid == blockDim.x - 1) carry = off + incl;
        __syncthreads();
    }
    if (tid == 0) seg_start[nseg] = carry;
}

// Identity expert: every received row goes back to its sender's back buffer,
// at the return address the dispatch stored beside it.  Rows are visited in
// a scattered order (row = q * kRowStride mod rows, a bijection because the
// stride is a prime larger than any row count), so at any moment the GPU's
// stores go to all senders at once instead of one sender's run of rows
// (measured on NVSwitch: 389 GB/s per GPU when all GPUs store to one peer at
// a time, 637 GB/s interleaved).  Each lane loads its whole share of a row
// into registers before storing any of it (a store to a peer pointer could
// alias the source, so the compiler would otherwise serialise every load
// behind the previous store).
constexpr int kReturnVPL = 8;  // 16-byte vectors per lane per pass: 4 KB rows in one pass
constexpr int64_t kRowStride = 2147483647;  // 2^31 - 1, prime

// Every CTA waits (bounded) for the senders' data flags.  seg_start ==
// nullptr (the one-call step): no receive kernel ran before this one, so the
// received rows are counted from the counts inbox.
__global__ void __launch_bounds__(256)
ep_return_identity_kernel(EpGeom g, char* const* __restrict__ peer, char* const* __restrict__ back,
                          const uint4* __restrict__ recv, const int64_t* __restrict__ ret,
                          const int32_t* __restrict__ seg_start, int nseg, EpSignal sig,
                          uint32_t* __restrict__ dev_status) {
    __shared__ int s_fail;
    __shared__ unsigned long long s_total;
    if (threadIdx.x == 0) {
        s_fail = 0;
        s_total = 0;
    }
    __syncthreads();
    pdl_wait_primary();
    const char* mine = peer[g.rank];
    wait_flags(reinterpret_cast<const uint64_t*>(mine + g.off_dflag), g.nranks, sig.epoch, g.timeout_ns, dev_status,
               &s_fail);
    int64_t total;
    if (seg_start) {
        total = seg_start[nseg];
    } else {
        // rows here: every sender's rows of the range's non-replicated
        // experts + this rank's own rows of the replicated ones
        const int32_t* inbox = reinterpret_cast<const int32_t*>(mine + g.off_inbox);
        unsigned long long part = 0;
        for (int i = threadIdx.x; i < g.nranks * g.E; i += blockDim.x) {
            const int s = i / g.E, e = i % g.E;
            const bool hot = ep_is_hot(g, e);
            if ((!hot && e >= g.first[g.rank] && e < g.first[g.rank + 1]) || (hot && s == g.rank))
                part += unsigned(inbox[i]);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
        if ((threadIdx.x & 31) == 0) atomicAdd(&s_total, part);
        __syncthreads();
        total = int64_t(s_total);
    }
    const int nvec = g.d / 8;
    const int lane = threadIdx.x & 31;
    const int64_t gw = int64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int64_t nw = int64_t(gridDim.x) * (blockDim.x >> 5);
    for (int64_t q = gw; q < total; q += nw) {
        const int64_t row = (q * kRowStride) % total;
        const int64_t r = ret[row];
        uint4* dst = reinterpret_cast<uint4*>(back[int(r >> 32)]) + int64_t(uint32_t(r)) * nvec;
        const uint4* src = recv + row * nvec;
        for (int c0 = 0; c0 < nvec; c0 += 32 * kReturnVPL) {
            uint4 v[kReturnVPL];
#pragma unroll
            for (int j = 0; j < kReturnVPL; ++j) {
                const int i = c0 + j * 32 + lane;
                v[j] = i < nvec ? ld_nc_v4_first(src + i) : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int j = 0; j < kReturnVPL; ++j) {
                const int i = c0 + j * 32 + lane;
                if (i < nvec) st_v4(dst + i, v[j]);
            }
        }
    }
    // the last CTA to finish raises the back flags of every sender (not
    // when a CTA gave up waiting for the rows: then the senders time out too)
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) ep_signal_done(sig, s_fail != 0);
}

// ------------------------------------------------------------------ host ----

static int sm_count_ep() {
    int dev = 0, n = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n > 0 ? n : 148;
}

static EpContext* as_ctx(void* c) {
    EpContext* ctx = static_cast<EpContext*>(c);
    return ctx;
}

}  // namespace moe_b200

using namespace moe_b200;

extern "C" {

int moe_b200_ep_create(int nranks, int rank, int E, int K, int d, int max_tokens, const int32_t* expert_first,
                       int timeout_ms, void** ctx_out) {
    if (!ctx_out || !expert_first) return fail(MOE_B200_ERR_INVALID_ARG, "ep_create: null pointer");
    if (nranks < 1 || nranks > kEpMaxRanks || rank < 0 || rank >= nranks || E < nranks || K < 1 || K > 32 ||
        d < 8 || d % 8 != 0 || max_tokens < 1 || timeout_ms < 1)
        return fail(MOE_B200_ERR_INVALID_ARG,
                    "ep_create: need 1<=nranks<=%d, 0<=rank<nranks, E>=nranks, 1<=K<=32, d%%8==0, "
                    "max_tokens>=1, timeout_ms>=1",
                    kEpMaxRanks);
    if (E > kEpMaxExperts) return fail(MOE_B200_ERR_UNSUPPORTED, "ep_create: E=%d above %d", E, kEpMaxExperts);
    if (expert_first[0] != 0 || expert_first[nranks] != E)
        return fail(MOE_B200_ERR_INVALID_ARG, "ep_create: expert_first must run from 0 to E");
    EpContext* ctx = new EpContext();
    EpGeom& g = ctx->g;
    g.nranks = nranks;
    g.rank = rank;
    g.E = E;
    g.K = K;
    g.d = d;
    g.max_tokens = max_tokens;
    for (int i = 0; i <= nranks; ++i) {
        g.first[i] = expert_first[i];
        if (i > 0 && expert_first[i] <= expert_first[i - 1]) {
            delete ctx;
            return fail(MOE_B200_ERR_INVALID_ARG, "ep_create: every rank must own at least one expert");
        }
    }
    std::memset(g.hot, 0, sizeof(g.hot));
    g.nhot = 0;
    g.lrange = g.first[rank + 1] - g.first[rank];
    g.off_cflag = 0;
    g.off_dflag = 8 * kEpMaxRanks;
    g.off_bflag = 16 * kEpMaxRanks;
    g.off_count = 24 * kEpMaxRanks;  // [0,2): return CTAs done / failed, [2,4): down-GEMM CTAs done / failed
    g.off_inbox = 4096;
    g.off_recv = g.off_inbox + al4k(size_t(nranks) * E * 4);
    g.recv_cap = int64_t(nranks) * max_tokens * K;
    g.off_ret = g.off_recv + al4k(size_t(g.recv_cap) * d * 2);
    g.off_back = g.off_ret + al4k(size_t(g.recv_cap) * 8);
    g.total = g.off_back + al4k(size_t(max_tokens) * K * d * 2);
    g.timeout_ns = uint64_t(timeout_ms) * 1000000ull;
    cudaError_t err = cudaGetDevice(&ctx->device);
    if (err == cudaSuccess) err = cudaMalloc(&ctx->region, g.total);
    if (err == cudaSuccess) err = cudaMemset(ctx->region, 0, g.total);
    if (err == cudaSuccess) err = cudaMalloc(&ctx->peer_dev, sizeof(char*) * kEpMaxRanks * 2);
    if (err == cudaSuccess) err = cudaMalloc(&ctx->seg, sizeof(int32_t) * 2 * (size_t(E) + 1));
    if (err != cudaSuccess) {
        if (ctx->region) cudaFree(ctx->region);
        if (ctx->peer_dev) cudaFree(ctx->peer_dev);
        delete ctx;
        return cuda_fail(err, "ep_create");
    }
    ctx->back_dev = ctx->peer_dev + kEpMaxRanks;
    *ctx_out = ctx;
    return MOE_B200_OK;
}

int moe_b200_ep_set_replicated(void* c, const int32_t* experts, int n) {
    EpContext* ctx = as_ctx(c);
    if (!ctx || (n > 0 && !experts)) return fail(MOE_B200_ERR_INVALID_ARG, "ep_set_replicated: null pointer");
    EpGeom& g = ctx->g;
    if (n < 0 || n > g.E) return fail(MOE_B200_ERR_INVALID_ARG, "ep_set_replicated: n=%d outside [0, E]", n);
    uint32_t hot[kEpMaxExperts / 32] = {};
    for (int i = 0; i < n; ++i) {
        const int e = experts[i];
        if (e < 0 || e >= g.E) return fail(MOE_B200_ERR_INVALID_ARG, "ep_set_replicated: expert %d outside [0, E)", e);
        if ((hot[e >> 5] >> (e & 31)) & 1u)
            return fail(MOE_B200_ERR_INVALID_ARG, "ep_set_replicated: expert %d listed twice", e);
        hot[e >> 5] |= 1u << (e & 31);
    }
    std::memcpy(g.hot, hot, sizeof(hot));
    g.nhot = n;
    int lr = 0;
    for (int e = g.first[g.rank]; e < g.first[g.rank + 1]; ++e)
        if (!ep_is_hot(g, e)) ++lr;
    g.lrange = lr;
    return MOE_B200_OK;
}

int moe_b200_ep_local_experts(void* c, int32_t* experts_out) {
    EpContext* ctx = as_ctx(c);
    if (!ctx) return -1;
    const EpGeom& g = ctx->g;
    int n = 0;
    for (int e = g.first[g.rank]; e < g.first[g.rank + 1]; ++e)
        if (!ep_is_hot(g, e)) {
            if (experts_out) experts_out[n] = e;
            ++n;
        }
    for (int e = 0; e < g.E; ++e)
        if (ep_is_hot(g, e)) {
            if (experts_out) experts_out[n] = e;
            ++n;
        }
    return n;
}

int moe_b200_ep_destroy(void* c) {
    EpContext* ctx = as_ctx(c);
    if (!ctx) return MOE_B200_OK;
    cudaDeviceSynchronize();
    for (int p = 0; p < ctx->g.nranks; ++p)
        if (ctx->opened[p]) cudaIpcCloseMemHandle(ctx->peer_host[p]);
    if (ctx->peer_dev) cudaFree(ctx->peer_dev);
    if (ctx->seg) cudaFree(ctx->seg);
    if (ctx->region) cudaFree(ctx->region);
    delete ctx;
    return MOE_B200_OK;
}

int moe_b200_ep_ipc_handle(void* c, void* handle_out) {
    EpContext* ctx = as_ctx(c);
    if (!ctx || !handle_out) return fail(MOE_B200_ERR_INVALID_ARG, "ep_ipc_handle: null pointer");
    cudaIpcMemHandle_t h;
    cudaError_t err = cudaIpcGetMemHandle(&h, ctx->region);
    if (err != cudaSuccess) return cuda_fail(err, "ep_ipc_handle");
    std::memcpy(handle_out, &h, sizeof(h));
    return MOE_B200_OK;
}

int moe_b200_ep_connect(void* c, const void* handles) {
    EpContext* ctx = as_ctx(c);
    if (!ctx || !handles) return fail(MOE_B200_ERR_INVALID_ARG, "ep_connect: null pointer");
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handles are 64 bytes");
    const EpGeom& g = ctx->g;
    char* back[kEpMaxRanks];
    for (int p = 0; p < g.nranks; ++p) {
        if (p == g.rank) {
            ctx->peer_host[p] = ctx->region;
        } else if (!ctx->opened[p]) {
            cudaIpcMemHandle_t h;
            std::memcpy(&h, static_cast<const char*>(handles) + 64 * p, 64);
            void* ptr = nullptr;
            cudaError_t err = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
            if (err != cudaSuccess) return cuda_fail(err, "ep_connect: cudaIpcOpenMemHandle");
            ctx->peer_host[p] = static_cast<char*>(ptr);
            ctx->opened[p] = true;
        }
        back[p] = ctx->peer_host[p] + g.off_back;
    }
    cudaError_t err = cudaMemcpy(ctx->peer_dev, ctx->peer_host, sizeof(char*) * g.nranks, cudaMemcpyHostToDevice);
    if (err == cudaSuccess) err = cudaMemcpy(ctx->back_dev, back, sizeof(char*) * g.nranks, cudaMemcpyHostToDevice);
    if (err != cudaSuccess) return cuda_fail(err, "ep_connect");
    ctx->connected = true;
    return MOE_B200_OK;
}

void* moe_b200_ep_recv_rows(void* c) {
    EpContext* ctx = as_ctx(c);
    return ctx ? ctx->region + ctx->g.off_recv : nullptr;
}

void* moe_b200_ep_back_rows(void* c) {
    EpContext* ctx = as_ctx(c);
    return ctx ? ctx->region + ctx->g.off_back : nullptr;
}

int64_t moe_b200_ep_recv_capacity(void* c) {
    EpContext* ctx = as_ctx(c);
    return ctx ? ctx->g.recv_cap : 0;
}

// Enqueue helpers shared by the stage entry points and moe_b200_ep_step.
static int ep_enqueue_dispatch(EpContext* ctx, uint64_t epoch, const void* emb, const int32_t* asgn,
                               const float* wts, int T, float* packed_weights, int32_t* perm,
                               int32_t* expert_count, int32_t* expert_start, int32_t* slot_pos, void* workspace,
                               size_t workspace_bytes, cudaStream_t s) {
    const EpGeom& g = ctx->g;
    if (T < 1 || T > g.max_tokens || !emb || !asgn || !perm || !expert_count || !expert_start || !slot_pos ||
        (packed_weights && !wts))
        return fail(MOE_B200_ERR_INVALID_ARG, "ep_dispatch: need 1 <= T <= max_tokens and all buffers");
    if (reinterpret_cast<uintptr_t>(emb) % 16 != 0)
        return fail(MOE_B200_ERR_INVALID_ARG, "ep_dispatch: rows must be 16-byte aligned");
    const PackPlan plan = plan_pack(T, g.K, g.E);
    if (!workspace || workspace_bytes < plan.total_bytes || reinterpret_cast<uintptr_t>(workspace) % 256)
        return fail(MOE_B200_ERR_WORKSPACE, "ep_dispatch: workspace of %zu bytes (256-aligned) needed",
                    plan.total_bytes);
    uint32_t* st = device_status_word();
    if (!st) return fail(MOE_B200_ERR_CUDA, "ep_dispatch: device status word unavailable");
    // the scan's last tile publishes the counts to every rank
    const EpPublish pub{ctx->peer_dev, g.off_inbox, g.off_cflag, g.rank, g.nranks, epoch};
    cudaError_t err = launch_route_scan(asgn, T, g.K, g.E, expert_count, expert_start, workspace, s, &pub);
    if (err == cudaSuccess) {
        char* base = static_cast<char*>(workspace);
        int grid = sm_count_ep() * 4;
        const int want = (T + 7) / 8;
        if (grid > want) grid = want;
        // the counts inbox goes to shared memory when it is small (N*E <= 4096)
        const int inbox_smem = int64_t(g.nranks) * g.E <= kInboxSmemMax ? 1 : 0;
        const size_t smem = size_t(g.E) * 16 + (inbox_smem ? size_t(g.nranks) * g.E * 4 : 0);
        cudaLaunchConfig_t cfg = pdl_config(dim3(grid), dim3(256), smem, s);
        cudaLaunchAttribute attr = pdl_attr();
        cfg.attrs = &attr;
        cfg.numAttrs = 1;
        err = cudaLaunchKernelEx(&cfg, ep_pack_dispatch_kernel, g, static_cast<char* const*>(ctx->peer_dev),
                                 static_cast<const uint4*>(emb), asgn, wts,
                                 static_cast<const int32_t*>(reinterpret_cast<int32_t*>(base + plan.rank_off)),
                                 static_cast<const int32_t*>(expert_start), T, packed_weights, perm, slot_pos,
                                 reinterpret_cast<WsHeader*>(base),
                                 reinterpret_cast<uint64_t*>(base + plan.status_off),
                                 size_t(plan.num_tiles) * size_t(g.E), epoch, st, inbox_smem);
    }
    if (err == cudaSuccess && epoch > ctx->epoch) ctx->epoch = epoch;
    return err == cudaSuccess ? MOE_B200_OK : cuda_fail(err, "ep_dispatch launch");
}

static int ep_enqueue_receive(EpContext* ctx, uint64_t epoch, int32_t* seg_start, int32_t* seg_expert,
                              bool wait_rows, cudaStream_t s) {
    if (!seg_start || !seg_expert) return fail(MOE_B200_ERR_INVALID_ARG, "ep_receive: null segment buffer");
    uint32_t* st = device_status_word();
    if (!st) return fail(MOE_B200_ERR_CUDA, "ep_receive: device status word unavailable");
    const int inbox_smem = int64_t(ctx->g.nranks) * ctx->g.E <= kInboxSmemMax ? 1 : 0;
    const size_t smem = inbox_smem ? size_t(ctx->g.nranks) * ctx->g.E * 4 : 0;
    ep_receive_kernel<<<1, 256, smem, s>>>(ctx->g, ctx->peer_dev, epoch, seg_start, seg_expert, st, inbox_smem,
                                           wait_rows ? 1 : 0);
    cudaError_t err = cudaGetLastError();
    return err == cudaSuccess ? MOE_B200_OK : cuda_fail(err, "ep_receive launch");
}

static EpSignal back_signal(EpContext* ctx, int which, uint64_t epoch) {
    const EpGeom& g = ctx->g;
    return EpSignal{ctx->peer_dev, g.off_bflag,
                    reinterpret_cast<uint32_t*>(ctx->region + g.off_count) + 2 * which, g.rank, g.nranks, epoch};
}

// seg_start == nullptr: the return kernel waits for the senders itself (no
// receive kernel before it).
static int ep_enqueue_return_identity(EpContext* ctx, uint64_t epoch, const int32_t* seg_start, cudaStream_t s) {
    const EpGeom& g = ctx->g;
    const int nseg = g.lrange + g.nhot;
    uint32_t* st = device_status_word();
    if (!st) return fail(MOE_B200_ERR_CUDA, "ep_return_identity: device status word unavailable");
    cudaLaunchConfig_t cfg = pdl_config(dim3(sm_count_ep() * 4), dim3(256), 0, s);
    cudaLaunchAttribute attr = pdl_attr();
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    cudaError_t err = cudaLaunchKernelEx(&cfg, ep_return_identity_kernel, g, static_cast<char* const*>(ctx->peer_dev),
                                         static_cast<char* const*>(ctx->back_dev),
                                         reinterpret_cast<const uint4*>(ctx->region + g.off_recv),
                                         reinterpret_cast<const int64_t*>(ctx->region + g.off_ret), seg_start, nseg,
                                         back_signal(ctx, 0, epoch), st);
    return err == cudaSuccess ? MOE_B200_OK : cuda_fail(err, "ep_return_identity launch");
}

static int ep_enqueue_ffn_return(EpContext* ctx, uint64_t epoch, const int32_t* seg_start,
                                 const int32_t* seg_expert, int I, const void* w_gate_up, const void* w_down,
                                 int dtype, void* h, cudaStream_t s) {
    const EpGeom& g = ctx->g;
    // One segment per local expert: the replicated ones first (this rank's
    // own rows, in place since its dispatch finished), then the range's
    // non-replicated ones.  GEMM 1 starts on the replicated segments and
    // its producers wait for every sender's data flag before the first
    // load of the others.  GEMM 2's epilogue stores every finished row
    // straight into the back buffer of the rank that sent it, at the return
    // address stored beside the row (scatter mode); its last CTA raises the
    // back flags.
    const EpSignal sig = back_signal(ctx, 1, epoch);
    const EpWait rows{reinterpret_cast<const uint64_t*>(ctx->region + g.off_dflag), g.nranks, epoch, g.timeout_ns};
    return grouped_swiglu_impl(ctx->region + g.off_recv, seg_start, seg_expert, g.lrange + g.nhot,
                               int(g.recv_cap), g.d, I, g.lrange + g.nhot, w_gate_up, w_down, dtype, h,
                               ctx->region + g.off_recv, s, ctx->back_dev,
                               reinterpret_cast<const int64_t*>(ctx->region + g.off_ret), nullptr, 0, &sig, &rows,
                               g.nhot);
}

static int ep_enqueue_combine(EpContext* ctx, uint64_t epoch, const float* packed_weights, const int32_t* slot_pos,
                              int T, int dtype, void* out, cudaStream_t s) {
    const EpGeom& g = ctx->g;
    if (T < 1 || T > g.max_tokens || !packed_weights || !slot_pos || !out)
        return fail(MOE_B200_ERR_INVALID_ARG, "ep_combine: need 1 <= T <= max_tokens and all buffers");
    if (dtype != MOE_B200_F16 && dtype != MOE_B200_BF16)
        return fail(MOE_B200_ERR_INVALID_ARG, "ep_combine: dtype %d is neither F16 nor BF16", dtype);
    // the unpermute's copy warps wait for every rank's back flag
    const EpWait wt{reinterpret_cast<const uint64_t*>(ctx->region + g.off_bflag), g.nranks, epoch, g.timeout_ns};
    cudaError_t err = launch_unpermute(ctx->region + g.off_back, packed_weights, slot_pos, T, g.K, g.d, dtype, out, s,
                                       &wt);
    return err == cudaSuccess ? MOE_B200_OK : cuda_fail(err, "ep_combine launch");
}

static EpContext* connected_ctx(void* c, const char* what) {
    EpContext* ctx = as_ctx(c);
    if (!ctx || !ctx->connected) {
        fail(MOE_B200_ERR_INVALID_ARG, "%s: context not connected", what);
        return nullptr;
    }
    return ctx;
}

int moe_b200_ep_dispatch(void* c, uint64_t epoch, const void* emb, const int32_t* asgn, const float* wts, int T,
                         float* packed_weights, int32_t* perm, int32_t* expert_count, int32_t* expert_start,
                         int32_t* slot_pos, void* workspace, size_t workspace_bytes, void* stream) {
    EpContext* ctx = connected_ctx(c, "ep_dispatch");
    if (!ctx) return MOE_B200_ERR_INVALID_ARG;
    return ep_enqueue_dispatch(ctx, epoch, emb, asgn, wts, T, packed_weights, perm, expert_count, expert_start,
                               slot_pos, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

int moe_b200_ep_receive(void* c, uint64_t epoch, int32_t* seg_start, int32_t* seg_expert, void* stream) {
    EpContext* ctx = connected_ctx(c, "ep_receive");
    if (!ctx) return MOE_B200_ERR_INVALID_ARG;
    // alone: the rows are in place when it ends, whatever expert follows
    return ep_enqueue_receive(ctx, epoch, seg_start, seg_expert, true, static_cast<cudaStream_t>(stream));
}

int moe_b200_ep_return_identity(void* c, uint64_t epoch, const int32_t* seg_start, void* stream) {
    EpContext* ctx = connected_ctx(c, "ep_return_identity");
    if (!ctx) return MOE_B200_ERR_INVALID_ARG;
    if (!seg_start) return fail(MOE_B200_ERR_INVALID_ARG, "ep_return_identity: null segment buffer");
    return ep_enqueue_return_identity(ctx, epoch, seg_start, static_cast<cudaStream_t>(stream));
}

int moe_b200_ep_ffn_return(void* c, uint64_t epoch, const int32_t* seg_start, const int32_t* seg_expert, int I,
                           const void* w_gate_up, const void* w_down, int dtype, void* h, void* stream) {
    EpContext* ctx = connected_ctx(c, "ep_ffn_return");
    if (!ctx) return MOE_B200_ERR_INVALID_ARG;
    if (!seg_start || !seg_expert) return fail(MOE_B200_ERR_INVALID_ARG, "ep_ffn_return: null segment buffer");
    return ep_enqueue_ffn_return(ctx, epoch, seg_start, seg_expert, I, w_gate_up, w_down, dtype, h,
                                 static_cast<cudaStream_t>(stream));
}

int moe_b200_ep_combine(void* c, uint64_t epoch, const float* packed_weights, const int32_t* slot_pos, int T,
                        int dtype, void* out, void* stream) {
    EpContext* ctx = connected_ctx(c, "ep_combine");
    if (!ctx) return MOE_B200_ERR_INVALID_ARG;
    return ep_enqueue_combine(ctx, epoch, packed_weights, slot_pos, T, dtype, out, static_cast<cudaStream_t>(stream));
}

int moe_b200_ep_step(void* c, const void* emb, const int32_t* asgn, const float* wts, int T, int I,
                     const void* w_gate_up, const void* w_down, int dtype, void* h, float* packed_weights,
                     int32_t* perm, int32_t* expert_count, int32_t* expert_start, int32_t* slot_pos,
                     void* workspace, size_t workspace_bytes, void* out, void* stream) {
    EpContext* ctx = connected_ctx(c, "ep_step");
    if (!ctx) return MOE_B200_ERR_INVALID_ARG;
    const EpGeom& g = ctx->g;
    if (!packed_weights) return fail(MOE_B200_ERR_INVALID_ARG, "ep_step: packed_weights is required");
    const bool identity = w_gate_up == nullptr && w_down == nullptr;
    if (!identity && (!w_gate_up || !w_down || !h || I < 1))
        return fail(MOE_B200_ERR_INVALID_ARG, "ep_step: the FFN needs w_gate_up, w_down, h and I >= 1");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const uint64_t epoch = ctx->epoch + 1;
    int32_t* seg_start = ctx->seg;                  // [E + 1]
    int32_t* seg_expert = seg_start + (g.E + 1);   // [E]
    int st = ep_enqueue_dispatch(ctx, epoch, emb, asgn, wts, T, packed_weights, perm, expert_count, expert_start,
                                 slot_pos, workspace, workspace_bytes, s);
    // identity: the return kernel waits for the senders itself (four launches
    // per step); the FFN needs the receive kernel's segment table
    // (the segment table from the counts; the gate/up GEMM waits for the rows)
    if (st == MOE_B200_OK && !identity) st = ep_enqueue_receive(ctx, epoch, seg_start, seg_expert, false, s);
    if (st == MOE_B200_OK)
        st = identity ? ep_enqueue_return_identity(ctx, epoch, nullptr, s)
                      : ep_enqueue_ffn_return(ctx, epoch, seg_start, seg_expert, I, w_gate_up, w_down, dtype, h, s);
    if (st == MOE_B200_OK) st = ep_enqueue_combine(ctx, epoch, packed_weights, slot_pos, T, dtype, out, s);
    return st;
}

uint64_t moe_b200_ep_epoch(void* c) {
    EpContext* ctx = as_ctx(c);
    return ctx ? ctx->epoch : 0;
}

}  // extern "C"
