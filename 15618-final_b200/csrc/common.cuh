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
//   [0, 256)          WsHeader: tile ticket, finished-tile counter, device
//                     condition bits
//   tile_status       num_tiles * E  u64 words of the decoupled look-back
//   rank              T*K int32: rank of slot (t, k) among the earlier slots
//                     routed to the same expert
// The route/scan kernel leaves ticket, counter and tile_status at zero when it
// finishes, so a workspace zero-filled once stays valid for every later call.
struct WsHeader {
    uint32_t ticket;
    uint32_t done;
    uint32_t status;
    uint32_t pad[61];
};
static_assert(sizeof(WsHeader) == 256, "header is one 256-byte block");

constexpr int kScanThreads = 256;           // route/scan CTA size (8 warps)
constexpr int kScanWarps = kScanThreads / 32;
constexpr int kSlotsPerWarpChunk = 32;
constexpr int kBaseTileSlots = kScanThreads * 8;  // 2048 slots per tile
constexpr size_t kMaxStatusBytes = size_t(16) << 20;

struct PackPlan {
    int tile_slots;   // slots per route/scan tile
    int num_tiles;
    size_t status_off, rank_off, total_bytes;
};

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// Tile size grows in powers of two only when the look-back status array would
// exceed kMaxStatusBytes (very large T*K times E).
inline PackPlan plan_pack(int T, int K, int E) {
    PackPlan p{};
    int64_t TK = int64_t(T) * K;
    int64_t tile = kBaseTileSlots;
    while (true) {
        int64_t nt = (TK + tile - 1) / tile;
        if (size_t(nt) * size_t(E) * 8 <= kMaxStatusBytes || tile >= (int64_t(1) << 24)) {
            p.tile_slots = int(tile);
            p.num_tiles = int(nt);
            break;
        }
        tile *= 2;
    }
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

}  // namespace moe_b200
