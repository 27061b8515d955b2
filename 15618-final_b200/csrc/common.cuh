// common.cuh -- device helpers and the workspace layout shared by the packing
// and combine kernels of libmoe_b200 (sm_100a).
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "moe_b200.h"

namespace moe_b200 {

// ---------------------------------------------------------------- layout ----
// Packing workspace (all offsets 256-byte aligned):
//   [0, 256)          WsHeader: tile ticket, device condition bits
//   tile_status       num_tiles * E  u64 words of the decoupled look-back
//   rank              T*K int32: rank of slot (t, k) among the earlier slots
//                     routed to the same expert
// pack_rows re-zeroes the ticket and tile_status after the route/scan kernel
// has finished, so a workspace zero-filled once stays valid for every later
// call.
struct WsHeader {
    uint32_t ticket;
    uint32_t status;
    uint32_t pad[62];
};
static_assert(sizeof(WsHeader) == 256, "header is one 256-byte block");

constexpr int kScanWarps = 8;                    // route/scan CTA: 8 warps
constexpr int kScanThreads = kScanWarps * 32;
#ifndef MOE_B200_SCAN_CHUNKS
#define MOE_B200_SCAN_CHUNKS 8
#endif
constexpr int kScanChunks = MOE_B200_SCAN_CHUNKS;  // 32-slot chunks per warp
constexpr int kTileSlots = kScanThreads * kScanChunks;  // 2048 slots per tile

struct PackPlan {
    int num_tiles;
    size_t status_off, rank_off, total_bytes;
};

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

inline PackPlan plan_pack(int T, int K, int E) {
    PackPlan p{};
    int64_t TK = int64_t(T) * K;
    p.num_tiles = int((TK + kTileSlots - 1) / kTileSlots);
    p.status_off = sizeof(WsHeader);
    p.rank_off = p.status_off + align256(size_t(p.num_tiles) * size_t(E) * 8);
    p.total_bytes = p.rank_off + align256(size_t(TK) * 4);
    return p;
}

// ------------------------------------------------------------ PTX helpers ----
__device__ __forceinline__ uint32_t lanemask_lt() {
    uint32_t m;
    asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
    return m;
}

__device__ __forceinline__ uint64_t ld_relaxed_u64(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_relaxed_u64(uint64_t* p, uint64_t v) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Read-only 16-byte load that does not allocate in L1 (streamed rows).
__device__ __forceinline__ uint4 ld_nc_v4(const uint4* p) {
    uint4 r;
    asm("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
        : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
        : "l"(p));
    return r;
}

__device__ __forceinline__ void st_v4(uint4* p, const uint4& v) {
    asm volatile("st.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y),
                 "r"(v.z), "r"(v.w)
                 : "memory");
}

// Programmatic dependent launch (PDL): the primary lets its dependent grid be
// scheduled early; the dependent waits for the primary's completion (and its
// memory) before touching what the primary writes.
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait_primary() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Upper bound on the polls of one cross-CTA wait (with a 64 ns back-off each,
// roughly 1 s); past it the kernel records MOE_B200_DEV_WAIT_TIMEOUT and
// moves on instead of spinning forever.
constexpr uint32_t kMaxPolls = 1u << 24;

// ------------------------------------------------ mbarrier / bulk copies ----
__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait for the phase with the given parity to complete: gives up
// after kWaitLimitNs of wall time and returns false.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (globaltimer_ns() - t0 > kWaitLimitNs) return false;
    }
}

// After an aborted pipeline, before a producer returns: the most recent load
// issued into every stage has landed (bounded wait), so no copy is still
// writing into shared memory when the CTA exits.  `issued` = stage fills
// issued.  (On the normal path the consumers waited for every fill.)
__device__ __forceinline__ void drain_stages(uint64_t* full, uint32_t issued, int stages) {
    for (uint32_t j = issued > uint32_t(stages) ? issued - uint32_t(stages) : 0u; j < issued; ++j)
        mbar_wait(full + j % uint32_t(stages), (j / uint32_t(stages)) & 1u);
}

// Bulk (non-tensor) copy global -> shared, completing on an mbarrier.  Both
// addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes,
                                         uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(smem_dst)),
        "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Bulk copy shared -> global, tracked by the issuing thread's bulk group.
__device__ __forceinline__ void bulk_s2g(void* gmem_dst, const void* smem_src, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gmem_dst),
                 "r"(smem_u32(smem_src)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until at most N committed bulk groups of this thread still READ shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
template <int N>
__device__ __forceinline__ void bulk_wait() {
    asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

uint32_t* device_status_word();  // status.cu

// ------------------------------------------- expert-parallel flag words ----
// System-scope acquire / release on epoch words that other GPUs read or write
// over NVLink (CUDA IPC mappings).
__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(uint64_t* p, uint64_t v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
// Orders this thread's earlier generic-proxy accesses (e.g. an acquire of a
// peer's flag) before its later async-proxy (cp.async.bulk) global accesses.
__device__ __forceinline__ void fence_proxy_async_global() {
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Count publication folded into the route/scan kernel (expert parallel):
// the tile that finishes the scan writes the final expert counts into row
// `rank` of every rank's counts inbox and raises every rank's counts flag
// [rank] to `epoch`.  peer == nullptr: no publication (single GPU).
struct EpPublish {
    char* const* peer;  // device array: every rank's region base, this address space
    size_t off_inbox, off_flag;
    int rank, nranks;
    uint64_t epoch;
};

// "Last CTA raises the flags": every CTA of a grid that stored rows into
// peers' buffers counts itself done in `counter`; the last one raises flag
// word [rank] at `flag_off` of every rank's region to `epoch`, unless some
// CTA reported a failure in `failed` (then no flag is raised and the peers'
// bounded waits time out and report it themselves).  peer == nullptr: off.
struct EpSignal {
    char* const* peer;
    size_t flag_off;
    uint32_t* counter;  // [0]: CTAs done, [1]: failure mark; both start and end at 0
    int rank, nranks;
    uint64_t epoch;
};

// Called by one thread per CTA after the CTA's peer stores were fenced
// system-wide and the CTA synchronised.
__device__ __forceinline__ void ep_signal_done(const EpSignal& sig, bool cta_failed) {
    if (cta_failed) atomicOr(sig.counter + 1, 1u);
    __threadfence();
    const uint32_t prev = atomicAdd(sig.counter, 1u);
    if (prev != gridDim.x * gridDim.y * gridDim.z - 1) return;
    __threadfence();
    const bool any_failed = atomicExch(sig.counter + 1, 0u) != 0u;
    sig.counter[0] = 0;
    if (any_failed) return;
    __threadfence_system();
    for (int p = 0; p < sig.nranks; ++p)
        st_release_sys(reinterpret_cast<uint64_t*>(sig.peer[p] + sig.flag_off) + sig.rank, sig.epoch);
}

// Bounded wait (in the kernel that consumes the peers' rows) for flag words
// [0, n) at `flags` to reach `epoch`.  flags == nullptr: no wait.
struct EpWait {
    const uint64_t* flags;
    int n;
    uint64_t epoch;
    uint64_t timeout_ns;
};

// After the route/scan grid has finished (PDL wait done): re-zero its ticket
// and look-back words so the workspace is ready for the next call.
__device__ __forceinline__ void rearm_scan_scratch(WsHeader* hdr, uint64_t* status, size_t words) {
    const size_t gt = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
    const size_t nt = size_t(gridDim.x) * blockDim.x;
    for (size_t i = gt; i < words; i += nt) status[i] = 0;
    if (gt == 0) hdr->ticket = 0;
}


// Launch configuration that lets the kernel start while the previous kernel
// in the stream finishes (programmatic dependent launch); the kernel must call
// pdl_wait_primary() before touching anything the previous kernel writes.
inline cudaLaunchConfig_t pdl_config(dim3 grid, dim3 block, size_t smem, cudaStream_t stream) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    return cfg;
}
inline cudaLaunchAttribute pdl_attr() {
    cudaLaunchAttribute a;
    a.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    a.val.programmaticStreamSerializationAllowed = 1;
    return a;
}

}  // namespace moe_b200
