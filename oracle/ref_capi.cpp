// ref_capi.cpp -- C entry points over the reference's own CPU oracle, so that
// Python tests can call it through ctypes.  TEST INFRASTRUCTURE ONLY.
//
// Built by oracle/Makefile together with the UNCHANGED reference sources
// src/common/cpu_reference.cpp (cpu_scatter :12-51, verify_scatter_outputs
// :61-178) into oracle/_ref/libref_cpu.so.  Nothing in the product links it.
#include "moe/cpu_reference.hpp"

#include <cstdint>

extern "C" {

void ref_cpu_scatter(const std::uint16_t* emb, const std::int32_t* asgn, const float* wts,
                     int T, int K, int E, int d,
                     std::uint16_t* packed, float* packed_w,
                     std::int32_t* expert_start, std::int32_t* expert_count,
                     std::int32_t* perm) {
    moe::cpu_scatter(emb, asgn, wts, T, K, E, d, packed, packed_w,
                     expert_start, expert_count, perm);
}

int ref_verify_scatter_outputs(const std::uint16_t* emb, const std::int32_t* asgn,
                               const float* wts, const std::uint16_t* packed,
                               const float* packed_w, const std::int32_t* expert_start,
                               const std::int32_t* expert_count, const std::int32_t* perm,
                               int T, int K, int E, int d) {
    return moe::verify_scatter_outputs(emb, asgn, wts, packed, packed_w, expert_start,
                                       expert_count, perm, T, K, E, d) ? 1 : 0;
}

}  // extern "C"
