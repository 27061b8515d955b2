// iscatter_b200.cpp -- the reference's C++ plugin boundary, moe::IScatter and
// moe::make_scatter (reference include/moe/scatter.cuh:28-65,
// src/scatter/factory.cu:11-18), implemented over the C ABI of libmoe_b200 so
// that programs written against that interface (verify, bench_scatter,
// bench_e2e, bench_ep) link against this library unchanged.
//
// Behaviour kept from the reference boundary:
//  - make_scatter returns nullptr for unknown names (factory.cu:17);
//  - workspace_bytes depends on the MoEParams only (bench_ep.cu:188 sizes the
//    scratch with a throw-away instance);
//  - run() enqueues on `stream` and may be called back to back without the
//    caller re-zeroing anything (bench_scatter.cu:235-239);
//  - errors print one line and exit(1), as MOE_CUDA_CHECK and the vec/csort
//    shape checks do (include/moe/utils.cuh:14-22, scatter_vec.cu:159-164).
// Changed on purpose: run() does not block the host.  ScatterTimings stays
// zero ("not measured", scatter.cuh:19) unless MOE_B200_STAGE_TIMING=1, in
// which case total_ms and gather_ms are measured with one event pair and one
// synchronisation.
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <string>

#include "moe/scatter.cuh"
#include "moe_b200.h"

namespace moe {

// Reference strategies: present only when the reference's strategy objects
// are linked into the same program (weak references otherwise stay null).
std::unique_ptr<IScatter> make_atomic_scatter() __attribute__((weak));
std::unique_ptr<IScatter> make_sort_scatter() __attribute__((weak));
std::unique_ptr<IScatter> make_warp_scatter() __attribute__((weak));
std::unique_ptr<IScatter> make_vec_scatter() __attribute__((weak));
std::unique_ptr<IScatter> make_csort_scatter() __attribute__((weak));

namespace {

[[noreturn]] void die(const char* what, int status) {
    std::fprintf(stderr, "b200 scatter: %s failed: %s (%s)\n", what,
                 moe_b200_status_string(status), moe_b200_last_error());
    std::exit(1);
}

bool stage_timing_requested() {
    const char* v = std::getenv("MOE_B200_STAGE_TIMING");
    return v && v[0] == '1';
}

class B200Scatter final : public IScatter {
public:
    const char* name() const override { return "b200"; }

    std::size_t workspace_bytes(const MoEParams& p) const override {
        return moe_b200_pack_workspace_bytes(p.T, p.K, p.E);
    }

    ScatterTimings run(const __half* d_emb, const int32_t* d_asgn, const float* d_wts,
                       MoEBuffers& bufs, const MoEParams& p, cudaStream_t stream) override {
        // A workspace seen for the first time (or with a new shape) is zero-filled
        // once; every pack call leaves it zero-filled for the next.
        if (bufs.strategy_ws != ws_ || bufs.strategy_ws_bytes != ws_bytes_ || p.T != T_ ||
            p.K != K_ || p.E != E_) {
            int st = moe_b200_workspace_init(bufs.strategy_ws, bufs.strategy_ws_bytes, stream);
            if (st != MOE_B200_OK) die("workspace init", st);
            ws_ = bufs.strategy_ws;
            ws_bytes_ = bufs.strategy_ws_bytes;
            T_ = p.T; K_ = p.K; E_ = p.E;
        }
        ScatterTimings t;
        cudaEvent_t ev[2] = {nullptr, nullptr};
        const bool timing = stage_timing_requested();
        if (timing) {
            cudaEventCreate(&ev[0]);
            cudaEventCreate(&ev[1]);
            cudaEventRecord(ev[0], stream);
        }
        int st = moe_b200_pack(d_emb, d_asgn, d_wts, p.T, p.K, p.E, p.d_model, bufs.packed,
                               bufs.packed_weights, bufs.perm, bufs.expert_count,
                               bufs.expert_start, nullptr, bufs.strategy_ws,
                               bufs.strategy_ws_bytes, stream);
        if (st != MOE_B200_OK) die("pack", st);
        if (timing) {
            cudaEventRecord(ev[1], stream);
            cudaEventSynchronize(ev[1]);
            cudaEventElapsedTime(&t.total_ms, ev[0], ev[1]);
            t.gather_ms = t.total_ms;
            cudaEventDestroy(ev[0]);
            cudaEventDestroy(ev[1]);
        }
        return t;
    }

private:
    void* ws_ = nullptr;
    std::size_t ws_bytes_ = 0;
    int T_ = -1, K_ = -1, E_ = -1;
};

}  // namespace

std::unique_ptr<IScatter> make_b200_scatter() { return std::make_unique<B200Scatter>(); }

std::unique_ptr<IScatter> make_scatter(const std::string& name) {
    if (name == "b200") return make_b200_scatter();
    if (name == "atomic") return make_atomic_scatter ? make_atomic_scatter() : nullptr;
    if (name == "sort") return make_sort_scatter ? make_sort_scatter() : nullptr;
    if (name == "warp") return make_warp_scatter ? make_warp_scatter() : nullptr;
    if (name == "vec") return make_vec_scatter ? make_vec_scatter() : nullptr;
    if (name == "csort") return make_csort_scatter ? make_csort_scatter() : nullptr;
    return nullptr;
}

}  // namespace moe
