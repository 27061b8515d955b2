// include/moe/types.h -- the plain-data boundary types of the MoE token-packing
// interface.  These declarations must stay layout-identical to the reference's
// include/moe/types.h:18-42 (MoEParams, MoEBuffers, Distribution): callers that
// were built against that header pass these structs by reference into
// moe::IScatter::run implemented by libmoe_b200.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_fp16.h>

namespace moe {

/// Problem sizes of one MoE layer pass.
struct MoEParams {
    int T;        ///< tokens
    int K;        ///< experts per token (top-K)
    int E;        ///< experts
    int d_model;  ///< hidden width (16-bit elements per token row)
    int d_ffn;    ///< expert inner width (unused by the packing step)
};

/// Caller-owned device buffers the packing step fills.
struct MoEBuffers {
    __half*  packed;          ///< [T*K, d_model] rows grouped by expert
    float*   packed_weights;  ///< [T*K] routing weight of each packed row
    int32_t* perm;            ///< [T*K] source token of each packed row
    int32_t* expert_count;    ///< [E]   rows per expert
    int32_t* expert_start;    ///< [E+1] first row of each expert; [E] = T*K
    void*    strategy_ws;     ///< scratch of workspace_bytes() bytes
    size_t   strategy_ws_bytes;
};

/// Routing distribution tag used by benchmark harnesses.
enum class Distribution { Uniform, Zipf };

}  // namespace moe
