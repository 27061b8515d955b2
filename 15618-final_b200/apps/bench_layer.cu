// bench_layer.cu -- C++ harness of one MoE layer through the C ABI only
// (include/moe_b200.h): router -> pack -> grouped SwiGLU FFN -> unpermute on
// one stream.  It is the counterpart of the reference's single-GPU layer
// harness, apps/bench_e2e.cu run_e2e (:218-329: fused_route_kernel ->
// IScatter::run -> per-expert cublasHgemm loop -> unpack_combine_kernel),
// for C/C++ callers of the new entry points the reference keeps inline in its
// apps.  Unlike run_e2e, a step never synchronises the host (the reference
// copies the expert counts to the host before its GEMM loop, :259-266).
//
// Each stage is timed with CUDA events on the launching stream, L2 is flushed
// (256 MiB memset) before every step, and the last step's outputs are checked
// on the host: routing invariants, the packing contract of moe::cpu_scatter
// (expert-major, ascending token within an expert, exclusive starts), the
// inverse permutation, and the layer output of a few tokens against an fp64
// host evaluation of the same SwiGLU experts.
//
//   bench_layer [--T 16384] [--d 2048] [--E 60] [--K 4] [--I 1408]
//               [--dtype bf16|fp16] [--iters 20] [--warmup 3] [--seed 1]
// Prints a table and one JSON line; exits non-zero on any failed check.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "moe_b200.h"

namespace {

struct Args {
    int T = 16384, d = 2048, E = 60, K = 4, I = 1408, iters = 20, warmup = 3;
    unsigned seed = 1;
    int dtype = MOE_B200_BF16;
};

[[noreturn]] void die(const char* what, const char* detail) {
    std::fprintf(stderr, "bench_layer: %s: %s\n", what, detail);
    std::exit(1);
}

void ck(cudaError_t e, const char* what) {
    if (e != cudaSuccess) die(what, cudaGetErrorString(e));
}

void ckm(int st, const char* what) {
    if (st != MOE_B200_OK) die(what, moe_b200_last_error());
}

Args parse(int argc, char** argv) {
    Args a;
    for (int i = 1; i + 1 < argc; i += 2) {
        const std::string k = argv[i];
        const char* v = argv[i + 1];
        if (k == "--T") a.T = std::atoi(v);
        else if (k == "--d") a.d = std::atoi(v);
        else if (k == "--E") a.E = std::atoi(v);
        else if (k == "--K") a.K = std::atoi(v);
        else if (k == "--I") a.I = std::atoi(v);
        else if (k == "--iters") a.iters = std::atoi(v);
        else if (k == "--warmup") a.warmup = std::atoi(v);
        else if (k == "--seed") a.seed = unsigned(std::strtoul(v, nullptr, 10));
        else if (k == "--dtype") a.dtype = std::string(v) == "fp16" ? MOE_B200_F16 : MOE_B200_BF16;
        else die("unknown option", k.c_str());
    }
    if (a.T < 1 || a.d < 16 || a.E < 1 || a.K < 1 || a.K > std::min(8, a.E) || a.I < 16 || a.iters < 1 ||
        a.warmup < 0)
        die("arguments", "need T>=1, d>=16, 1<=K<=min(8,E), I>=16, iters>=1");
    return a;
}

// Uniform values in [-r, r) from a 32-bit linear congruential generator.
struct Lcg {
    uint32_t s;
    float next(float r) {
        s = s * 1664525u + 1013904223u;
        return (float(s >> 8) * (1.0f / 16777216.0f) * 2.0f - 1.0f) * r;
    }
};

uint16_t to16(float f, int dtype) {
    uint16_t h;
    if (dtype == MOE_B200_BF16) {
        __nv_bfloat16 b = __float2bfloat16(f);
        std::memcpy(&h, &b, 2);
    } else {
        __half b = __float2half(f);
        std::memcpy(&h, &b, 2);
    }
    return h;
}

float from16(uint16_t h, int dtype) {
    if (dtype == MOE_B200_BF16) {
        __nv_bfloat16 b;
        std::memcpy(&b, &h, 2);
        return __bfloat162float(b);
    }
    __half b;
    std::memcpy(&b, &h, 2);
    return __half2float(b);
}

std::vector<uint16_t> fill16(size_t n, uint32_t seed, float r, int dtype) {
    Lcg g{seed};
    std::vector<uint16_t> v(n);
    for (auto& x : v) x = to16(g.next(r), dtype);
    return v;
}

template <class T>
T* dmalloc(size_t n, const char* what) {
    void* p = nullptr;
    ck(cudaMalloc(&p, std::max<size_t>(n, 1) * sizeof(T)), what);
    return static_cast<T*>(p);
}

template <class T>
std::vector<T> to_host(const T* d, size_t n) {
    std::vector<T> h(n);
    ck(cudaMemcpy(h.data(), d, n * sizeof(T), cudaMemcpyDeviceToHost), "D2H");
    return h;
}

double median(std::vector<float> v) {
    std::sort(v.begin(), v.end());
    return v.size() % 2 ? v[v.size() / 2] : 0.5 * (v[v.size() / 2 - 1] + v[v.size() / 2]);
}

int g_failures = 0;
void expect(bool ok, const char* what) {
    if (!ok) {
        ++g_failures;
        std::fprintf(stderr, "CHECK FAILED: %s\n", what);
    }
}

}  // namespace

int main(int argc, char** argv) {
    const Args a = parse(argc, argv);
    const int T = a.T, d = a.d, E = a.E, K = a.K, I = a.I, dt = a.dtype;
    const int64_t TK = int64_t(T) * K;

    // ---- host inputs (seeded) ----
    std::vector<uint16_t> h_emb = fill16(size_t(T) * d, a.seed, 1.0f, dt);
    std::vector<float> h_gate(size_t(d) * E);
    {
        Lcg g{a.seed + 1};
        for (auto& x : h_gate) x = g.next(0.05f);
    }
    std::vector<uint16_t> h_wgu = fill16(size_t(E) * 2 * I * d, a.seed + 2, 0.03f, dt);
    std::vector<uint16_t> h_wdn = fill16(size_t(E) * d * I, a.seed + 3, 0.03f, dt);

    // ---- device buffers ----
    cudaStream_t st;
    ck(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking), "stream");
    uint16_t* emb = dmalloc<uint16_t>(size_t(T) * d, "emb");
    float* gate = dmalloc<float>(size_t(d) * E, "gate");
    uint16_t* wgu = dmalloc<uint16_t>(h_wgu.size(), "w_gate_up");
    uint16_t* wdn = dmalloc<uint16_t>(h_wdn.size(), "w_down");
    ck(cudaMemcpy(emb, h_emb.data(), h_emb.size() * 2, cudaMemcpyHostToDevice), "H2D emb");
    ck(cudaMemcpy(gate, h_gate.data(), h_gate.size() * 4, cudaMemcpyHostToDevice), "H2D gate");
    ck(cudaMemcpy(wgu, h_wgu.data(), h_wgu.size() * 2, cudaMemcpyHostToDevice), "H2D w_gate_up");
    ck(cudaMemcpy(wdn, h_wdn.data(), h_wdn.size() * 2, cudaMemcpyHostToDevice), "H2D w_down");

    const size_t rw_bytes = moe_b200_router_weights_bytes(d, E, dt);
    if (rw_bytes == 0) die("router_weights_bytes", "unsupported shape");
    void* rw = dmalloc<uint8_t>(rw_bytes, "router weights");
    ckm(moe_b200_router_prepare(gate, d, E, dt, rw, st), "router_prepare");

    int32_t* asgn = dmalloc<int32_t>(TK, "asgn");
    float* wts = dmalloc<float>(TK, "wts");
    uint16_t* packed = dmalloc<uint16_t>(size_t(TK) * d, "packed");
    float* pw = dmalloc<float>(TK, "packed_weights");
    int32_t* perm = dmalloc<int32_t>(TK, "perm");
    int32_t* count = dmalloc<int32_t>(E, "expert_count");
    int32_t* start = dmalloc<int32_t>(E + 1, "expert_start");
    int32_t* slot_pos = dmalloc<int32_t>(TK, "slot_pos");
    uint16_t* hmid = dmalloc<uint16_t>(size_t(TK) * I, "h");
    uint16_t* y = dmalloc<uint16_t>(size_t(TK) * d, "y");
    uint16_t* out = dmalloc<uint16_t>(size_t(T) * d, "out");
    const size_t ws_bytes = moe_b200_pack_workspace_bytes(T, K, E);
    void* ws = dmalloc<uint8_t>(ws_bytes, "workspace");
    ckm(moe_b200_workspace_init(ws, ws_bytes, st), "workspace_init");
    const size_t flush_bytes = size_t(256) << 20;
    void* flush = dmalloc<uint8_t>(flush_bytes, "L2 flush buffer");

    // ---- timed steps ----
    cudaEvent_t ev[5];
    for (auto& e : ev) ck(cudaEventCreate(&e), "event");
    std::vector<float> t_route, t_pack, t_ffn, t_unperm, t_layer;
    for (int it = 0; it < a.warmup + a.iters; ++it) {
        ck(cudaMemsetAsync(flush, it & 0xff, flush_bytes, st), "L2 flush");
        ck(cudaEventRecord(ev[0], st), "record");
        ckm(moe_b200_route(emb, T, d, E, K, dt, rw, asgn, wts, st), "route");
        ck(cudaEventRecord(ev[1], st), "record");
        ckm(moe_b200_pack(emb, asgn, wts, T, K, E, d, packed, pw, perm, count, start, slot_pos, ws, ws_bytes,
                          st),
            "pack");
        ck(cudaEventRecord(ev[2], st), "record");
        ckm(moe_b200_grouped_swiglu(packed, start, nullptr, E, int(TK), d, I, E, wgu, wdn, dt, hmid, y, st),
            "grouped_swiglu");
        ck(cudaEventRecord(ev[3], st), "record");
        ckm(moe_b200_unpermute(y, pw, slot_pos, T, K, d, dt, out, st), "unpermute");
        ck(cudaEventRecord(ev[4], st), "record");
        ck(cudaEventSynchronize(ev[4]), "sync");
        if (it < a.warmup) continue;
        float ms[4], total;
        for (int s = 0; s < 4; ++s) ck(cudaEventElapsedTime(&ms[s], ev[s], ev[s + 1]), "elapsed");
        ck(cudaEventElapsedTime(&total, ev[0], ev[4]), "elapsed");
        t_route.push_back(ms[0]);
        t_pack.push_back(ms[1]);
        t_ffn.push_back(ms[2]);
        t_unperm.push_back(ms[3]);
        t_layer.push_back(total);
    }
    int ws_st = 0, dev_st = 0;
    ckm(moe_b200_workspace_status(ws, ws_bytes, st, &ws_st), "workspace_status");
    ckm(moe_b200_device_status(st, &dev_st), "device_status");
    expect(ws_st == 0, "pack workspace reports no device-side condition");
    expect(dev_st == 0, "router / FFN / unpermute report no device-side condition");

    // ---- host checks on the last step ----
    const auto h_asgn = to_host(asgn, TK);
    const auto h_wts = to_host(wts, TK);
    const auto h_count = to_host(count, E);
    const auto h_start = to_host(start, E + 1);
    const auto h_perm = to_host(perm, TK);
    const auto h_slot = to_host(slot_pos, TK);
    const auto h_pw = to_host(pw, TK);
    const auto h_out = to_host(out, size_t(T) * d);

    bool route_ok = true;
    std::vector<int64_t> hist(E, 0);
    for (int t = 0; t < T; ++t) {
        float wsum = 0.f;
        for (int k = 0; k < K; ++k) {
            const int e = h_asgn[size_t(t) * K + k];
            const float w = h_wts[size_t(t) * K + k];
            if (e < 0 || e >= E || !(w > 0.f) || w > 1.f) { route_ok = false; continue; }
            if (k > 0 && w > h_wts[size_t(t) * K + k - 1]) route_ok = false;  // descending
            for (int j = 0; j < k; ++j)
                if (h_asgn[size_t(t) * K + j] == e) route_ok = false;           // distinct experts
            ++hist[e];
            wsum += w;
        }
        if (wsum > 1.0001f) route_ok = false;
    }
    expect(route_ok, "router: experts in range and distinct per token, weights in (0, 1], descending");

    bool pack_ok = h_start[0] == 0 && h_start[E] == TK;
    for (int e = 0; e < E && pack_ok; ++e) {
        pack_ok = h_count[e] == hist[e] && h_start[e + 1] == h_start[e] + h_count[e];
        for (int64_t p = h_start[e] + 1; pack_ok && p < h_start[e + 1]; ++p)
            pack_ok = h_perm[p] > h_perm[p - 1];                                  // stable within expert
    }
    expect(pack_ok, "pack: counts match the routing, exclusive starts, ascending tokens within each expert");
    bool inv_ok = true;
    for (int t = 0; t < T && inv_ok; ++t)
        for (int k = 0; k < K && inv_ok; ++k) {
            const int64_t p = h_slot[size_t(t) * K + k];
            inv_ok = p >= 0 && p < TK && h_perm[p] == t &&
                     p >= h_start[h_asgn[size_t(t) * K + k]] && p < h_start[h_asgn[size_t(t) * K + k] + 1] &&
                     h_pw[p] == h_wts[size_t(t) * K + k];
        }
    expect(inv_ok, "pack: slot_pos is the inverse of perm, rows land in their expert's segment");

    bool finite = true;
    for (uint16_t v : h_out) finite = finite && std::isfinite(from16(v, dt));
    expect(finite, "layer output is finite");

    // fp64 host evaluation of a few tokens: out[t] = sum_k w * down(silu(gate) * up)
    const int probe[4] = {0, T / 3, (2 * T) / 3, T - 1};
    double worst = 0.0;
    std::vector<double> x(d), hbuf(I), acc(d);
    for (int pi = 0; pi < 4; ++pi) {
        const int t = probe[pi];
        for (int i = 0; i < d; ++i) x[i] = from16(h_emb[size_t(t) * d + i], dt);
        std::fill(acc.begin(), acc.end(), 0.0);
        for (int k = 0; k < K; ++k) {
            const int e = h_asgn[size_t(t) * K + k];
            const double w = h_wts[size_t(t) * K + k];
            const uint16_t* wg = h_wgu.data() + size_t(e) * 2 * I * d;
            const uint16_t* wd = h_wdn.data() + size_t(e) * d * I;
            for (int j = 0; j < I; ++j) {
                double g = 0, u = 0;
                for (int i = 0; i < d; ++i) {
                    g += x[i] * from16(wg[size_t(j) * d + i], dt);
                    u += x[i] * from16(wg[size_t(I + j) * d + i], dt);
                }
                hbuf[j] = g / (1.0 + std::exp(-g)) * u;
            }
            for (int c = 0; c < d; ++c) {
                double s = 0;
                for (int j = 0; j < I; ++j) s += hbuf[j] * from16(wd[size_t(c) * I + j], dt);
                acc[c] += w * s;
            }
        }
        double scale = 0;
        for (int c = 0; c < d; ++c) scale = std::max(scale, std::fabs(acc[c]));
        for (int c = 0; c < d; ++c)
            worst = std::max(worst, std::fabs(from16(h_out[size_t(t) * d + c], dt) - acc[c]) / (scale + 1e-30));
    }
    // h and y are rounded to 16 bits once each, the output once more: a few
    // units of the format's epsilon relative to the row's largest value.
    const double tol = dt == MOE_B200_BF16 ? 3e-2 : 4e-3;
    expect(worst <= tol, "layer output of 4 tokens matches an fp64 host evaluation");

    // ---- report ----
    const double flops = 6.0 * double(TK) * d * I;
    const double r = median(t_route), pk = median(t_pack), f = median(t_ffn), u = median(t_unperm),
                 l = median(t_layer);
    std::printf("bench_layer  T=%d d=%d E=%d K=%d I=%d %s  (median of %d steps, L2 flushed)\n", T, d, E, K, I,
                dt == MOE_B200_BF16 ? "bf16" : "fp16", a.iters);
    std::printf("  route      %9.3f ms\n  pack       %9.3f ms\n  ffn        %9.3f ms  (%.0f TFLOP/s)\n"
                "  unpermute  %9.3f ms\n  layer      %9.3f ms\n",
                r, pk, f, flops / (f * 1e-3) / 1e12, u, l);
    std::printf("  checks: %s (output vs fp64 host, worst %.2e of the row max)\n",
                g_failures ? "FAIL" : "pass", worst);
    std::printf("{\"harness\": \"bench_layer\", \"T\": %d, \"d\": %d, \"E\": %d, \"K\": %d, \"I\": %d, "
                "\"dtype\": \"%s\", \"route_ms\": %.4f, \"pack_ms\": %.4f, \"ffn_ms\": %.4f, "
                "\"unpermute_ms\": %.4f, \"layer_ms\": %.4f, \"ffn_tflops\": %.1f, \"max_rel_err\": %.3e, "
                "\"checks\": \"%s\"}\n",
                T, d, E, K, I, dt == MOE_B200_BF16 ? "bf16" : "fp16", r, pk, f, u, l, flops / (f * 1e-3) / 1e12,
                worst, g_failures ? "fail" : "pass");

    for (auto& e : ev) cudaEventDestroy(e);
    for (void* p : {(void*)emb, (void*)gate, (void*)wgu, (void*)wdn, rw, (void*)asgn, (void*)wts, (void*)packed,
                    (void*)pw, (void*)perm, (void*)count, (void*)start, (void*)slot_pos, (void*)hmid, (void*)y,
                    (void*)out, ws, flush})
        cudaFree(p);
    cudaStreamDestroy(st);
    return g_failures ? 1 : 0;
}
