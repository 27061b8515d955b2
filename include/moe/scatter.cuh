// include/moe/scatter.cuh -- the strategy interface of the MoE packing step.
// Declaration-compatible with the reference's include/moe/scatter.cuh:20-65
// (ScatterTimings, IScatter, make_*_scatter, make_scatter) so that code built
// against it links unchanged against libmoe_b200.
//
// libmoe_b200 defines:
//   make_b200_scatter()   the sm_100a packing strategy ("b200")
//   make_scatter(name)    "b200" -> the strategy above; the reference strategy
//                         names ("atomic", "sort", "warp", "vec", "csort")
//                         resolve to the reference implementations when those
//                         are linked into the same program, else nullptr;
//                         unknown names -> nullptr.
#pragma once

#include "types.h"
#include <cuda_runtime.h>
#include <cstddef>
#include <memory>
#include <string>

namespace moe {

/// Per-stage times of one run(); 0 means "not measured".  The b200 strategy
/// measures nothing by default, so run() never blocks the host.
struct ScatterTimings {
    float count_ms  = 0.f;
    float prefix_ms = 0.f;
    float sort_ms   = 0.f;
    float gather_ms = 0.f;
    float total_ms  = 0.f;
};

class IScatter {
public:
    virtual ~IScatter() = default;
    virtual const char* name() const = 0;
    /// Scratch bytes for problem p; depends on p only.
    virtual std::size_t workspace_bytes(const MoEParams& p) const = 0;
    /// Packs d_emb [T, d_model] by expert into bufs, enqueued on `stream`.
    virtual ScatterTimings run(const __half*  d_emb,
                               const int32_t* d_asgn,
                               const float*   d_wts,
                               MoEBuffers&    bufs,
                               const MoEParams& p,
                               cudaStream_t   stream) = 0;
};

std::unique_ptr<IScatter> make_atomic_scatter();
std::unique_ptr<IScatter> make_sort_scatter();
std::unique_ptr<IScatter> make_warp_scatter();
std::unique_ptr<IScatter> make_vec_scatter();
std::unique_ptr<IScatter> make_csort_scatter();
std::unique_ptr<IScatter> make_b200_scatter();

std::unique_ptr<IScatter> make_scatter(const std::string& name);

}  // namespace moe
