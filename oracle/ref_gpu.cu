// ref_gpu.cu -- C entry points over the reference's own GPU routing and combine
// kernels, so golden vectors can be produced by the reference code itself.
// TEST INFRASTRUCTURE ONLY: nothing in the product links it.
//
// The reference keeps these kernels in an anonymous namespace inside an app
// (apps/bench_e2e.cu:51-152: gate_kernel, softmax_kernel, topk_kernel,
// fused_route_kernel, unpack_combine_kernel, f32_to_f16_kernel), so the app
// source is compiled UNCHANGED inside this translation unit (its main()
// renamed) and the launchers below use the reference's own launch shapes
// (apps/bench_e2e.cu:235-255 for the routers, :304-313 for the combine), and
// the whole run_e2e layer is exported for expert-FFN golden vectors.
// Built by `make -C oracle ref-gpu` into oracle/_ref/libref_gpu.so together
// with the unchanged reference library sources the app links
// (Makefile:97-98 of the reference).
//
// Every function takes HOST pointers, allocates its own device buffers,
// synchronises, and returns a cudaError_t value (0 = success).
#define main moe_ref_bench_e2e_main
#include "bench_e2e.cu"
#undef main

#include <cstdint>
#include <cstring>

namespace {

template <class T>
cudaError_t to_dev(T** d, const T* h, std::size_t n) {
    cudaError_t e = cudaMalloc(reinterpret_cast<void**>(d), n * sizeof(T) + 16);
    if (e != cudaSuccess || h == nullptr) return e;
    return cudaMemcpy(*d, h, n * sizeof(T), cudaMemcpyHostToDevice);
}

template <class T>
cudaError_t to_host(T* h, const T* d, std::size_t n) {
    return cudaMemcpy(h, d, n * sizeof(T), cudaMemcpyDeviceToHost);
}

}  // namespace

extern "C" {

// include/moe/fp16_host.hpp:22-39, the reference's deterministic input fills.
void ref_fill_random_half(std::uint16_t* buf, std::size_t n, std::uint32_t seed, float half_range) {
    moe::fill_random_half(buf, n, seed, half_range);
}

void ref_fill_random_float(float* buf, std::size_t n, std::uint32_t seed, float half_range) {
    moe::fill_random_float(buf, n, seed, half_range);
}

// fused_route_kernel (apps/bench_e2e.cu:95-130), launched as at :238-240:
// one CTA per token, E threads, E floats of dynamic shared memory.
int ref_gpu_fused_route(const std::uint16_t* emb, const float* w_gate, int T, int K, int E, int d,
                        std::int32_t* asgn, float* wts) {
    __half* d_emb = nullptr;
    float *d_w = nullptr, *d_wts = nullptr;
    std::int32_t* d_asgn = nullptr;
    cudaError_t e = to_dev(&d_emb, reinterpret_cast<const __half*>(emb), (std::size_t)T * d);
    if (!e) e = to_dev(&d_w, w_gate, (std::size_t)d * E);
    if (!e) e = to_dev<std::int32_t>(&d_asgn, nullptr, (std::size_t)T * K);
    if (!e) e = to_dev<float>(&d_wts, nullptr, (std::size_t)T * K);
    if (!e) {
        fused_route_kernel<<<T, E, E * sizeof(float)>>>(d_emb, d_w, T, K, E, d, d_asgn, d_wts);
        e = cudaGetLastError();
    }
    if (!e) e = cudaDeviceSynchronize();
    if (!e) e = to_host(asgn, d_asgn, (std::size_t)T * K);
    if (!e) e = to_host(wts, d_wts, (std::size_t)T * K);
    cudaFree(d_emb); cudaFree(d_w); cudaFree(d_asgn); cudaFree(d_wts);
    return (int)e;
}

// gate_kernel -> softmax_kernel -> topk_kernel (apps/bench_e2e.cu:52-93),
// launched as at :243-254 with 256-thread blocks; also returns the
// intermediate logits and probabilities [T, E].  topk_kernel holds E <= 128.
int ref_gpu_naive_route(const std::uint16_t* emb, const float* w_gate, int T, int K, int E, int d,
                        float* logits, float* probs, std::int32_t* asgn, float* wts) {
    const int blk = 256;
    __half* d_emb = nullptr;
    float *d_w = nullptr, *d_logits = nullptr, *d_probs = nullptr, *d_wts = nullptr;
    std::int32_t* d_asgn = nullptr;
    cudaError_t e = to_dev(&d_emb, reinterpret_cast<const __half*>(emb), (std::size_t)T * d);
    if (!e) e = to_dev(&d_w, w_gate, (std::size_t)d * E);
    if (!e) e = to_dev<float>(&d_logits, nullptr, (std::size_t)T * E);
    if (!e) e = to_dev<float>(&d_probs, nullptr, (std::size_t)T * E);
    if (!e) e = to_dev<std::int32_t>(&d_asgn, nullptr, (std::size_t)T * K);
    if (!e) e = to_dev<float>(&d_wts, nullptr, (std::size_t)T * K);
    if (!e) {
        gate_kernel<<<(T * E + blk - 1) / blk, blk>>>(d_emb, d_w, d_logits, T, E, d);
        softmax_kernel<<<(T + blk - 1) / blk, blk>>>(d_logits, d_probs, T, E);
        topk_kernel<<<(T + blk - 1) / blk, blk>>>(d_probs, d_asgn, d_wts, T, K, E);
        e = cudaGetLastError();
    }
    if (!e) e = cudaDeviceSynchronize();
    if (!e) e = to_host(logits, d_logits, (std::size_t)T * E);
    if (!e) e = to_host(probs, d_probs, (std::size_t)T * E);
    if (!e) e = to_host(asgn, d_asgn, (std::size_t)T * K);
    if (!e) e = to_host(wts, d_wts, (std::size_t)T * K);
    cudaFree(d_emb); cudaFree(d_w); cudaFree(d_logits); cudaFree(d_probs);
    cudaFree(d_asgn); cudaFree(d_wts);
    return (int)e;
}

// unpack_combine_kernel + f32_to_f16_kernel (apps/bench_e2e.cu:136-152) after
// zeroing the fp32 accumulator, launched as at :304-313 (one CTA of 256
// threads per packed row).  Returns the fp32 sums and the fp16 output.
int ref_gpu_unpack_combine(const std::uint16_t* y, const float* packed_w, const std::int32_t* perm,
                           int TK, int T, int d, float* out32, std::uint16_t* out16) {
    const int blk = 256;
    __half *d_y = nullptr, *d_out16 = nullptr;
    float *d_pw = nullptr, *d_out32 = nullptr;
    std::int32_t* d_perm = nullptr;
    cudaError_t e = to_dev(&d_y, reinterpret_cast<const __half*>(y), (std::size_t)TK * d);
    if (!e) e = to_dev(&d_pw, packed_w, (std::size_t)TK);
    if (!e) e = to_dev(&d_perm, perm, (std::size_t)TK);
    if (!e) e = to_dev<float>(&d_out32, nullptr, (std::size_t)T * d);
    if (!e) e = to_dev<__half>(&d_out16, nullptr, (std::size_t)T * d);
    if (!e) {
        moe::device_zero_async(d_out32, (std::size_t)T * d, 0);
        unpack_combine_kernel<<<TK, blk>>>(d_y, d_pw, d_perm, d_out32, TK, d);
        f32_to_f16_kernel<<<(T * d + blk - 1) / blk, blk>>>(d_out32, d_out16, T * d);
        e = cudaGetLastError();
    }
    if (!e) e = cudaDeviceSynchronize();
    if (!e) e = to_host(out32, d_out32, (std::size_t)T * d);
    if (!e) e = to_host(reinterpret_cast<__half*>(out16), d_out16, (std::size_t)T * d);
    cudaFree(d_y); cudaFree(d_pw); cudaFree(d_perm); cudaFree(d_out32); cudaFree(d_out16);
    return (int)e;
}

// The reference's whole single-GPU MoE layer, run_e2e (apps/bench_e2e.cu:
// 218-329) unchanged: router (fused_route_kernel when fused != 0, else the
// gate/softmax/top-K chain), the IScatter strategy `strategy` from the
// reference's own factory (src/scatter/factory.cu), the per-expert
// cublasHgemm up/down loop with d_ffn = p.d_ffn, and the atomic combine.
// Buffers come from the app's allocate_e2e (:192-215).  Inputs: emb [T, d]
// fp16, w_gate [d, E] fp32, w1 [E, d, F] and w2 [E, F, d] fp16.  Outputs
// (host): assignments / routing weights [T, K], perm / packed weights [T*K],
// expert start / count [E], the expert intermediate mid [T*K, F], the expert
// outputs y [T*K, d] in packed order and the combined output [T, d].
int ref_gpu_moe_layer(const std::uint16_t* emb, const float* w_gate, const std::uint16_t* w1,
                      const std::uint16_t* w2, int T, int K, int E, int d, int F, const char* strategy, int fused,
                      std::int32_t* asgn, float* rwt, std::int32_t* perm, float* packed_w,
                      std::int32_t* expert_start, std::int32_t* expert_count, std::uint16_t* mid,
                      std::uint16_t* y, std::uint16_t* out) {
    moe::MoEParams p{T, K, E, d, F};
    const std::size_t TK = (std::size_t)T * K;
    auto scatter = moe::make_scatter(strategy);
    if (!scatter) return (int)cudaErrorInvalidValue;
    __half *d_emb = nullptr, *d_w1 = nullptr, *d_w2 = nullptr;
    float* d_gate = nullptr;
    cudaError_t e = to_dev(&d_emb, reinterpret_cast<const __half*>(emb), (std::size_t)T * d);
    if (!e) e = to_dev(&d_gate, w_gate, (std::size_t)d * E);
    if (!e) e = to_dev(&d_w1, reinterpret_cast<const __half*>(w1), (std::size_t)E * d * F);
    if (!e) e = to_dev(&d_w2, reinterpret_cast<const __half*>(w2), (std::size_t)E * F * d);
    if (e) return (int)e;
    cublasHandle_t cublas;
    if (cublasCreate(&cublas) != CUBLAS_STATUS_SUCCESS) return (int)cudaErrorUnknown;
    E2EBuffers b = allocate_e2e(p, scatter->workspace_bytes(p), /*naive=*/fused == 0);
    run_e2e(d_emb, d_gate, d_w1, d_w2, p, fused != 0, *scatter, b, cublas, 0);
    e = cudaDeviceSynchronize();
    if (!e) e = to_host(asgn, b.d_asgn, TK);
    if (!e) e = to_host(rwt, b.d_rwt, TK);
    if (!e) e = to_host(perm, b.scatter_bufs.perm, TK);
    if (!e) e = to_host(packed_w, b.scatter_bufs.packed_weights, TK);
    if (!e) e = to_host(expert_start, b.scatter_bufs.expert_start, (std::size_t)E);
    if (!e) e = to_host(expert_count, b.scatter_bufs.expert_count, (std::size_t)E);
    if (!e) e = to_host(reinterpret_cast<__half*>(mid), b.d_ffn_tmp, TK * F);
    if (!e) e = to_host(reinterpret_cast<__half*>(y), b.d_expert_out, TK * d);
    if (!e) e = to_host(reinterpret_cast<__half*>(out), b.d_output, (std::size_t)T * d);
    b.free();
    cublasDestroy(cublas);
    cudaFree(d_emb); cudaFree(d_gate); cudaFree(d_w1); cudaFree(d_w2);
    return (int)e;
}

}  // extern "C"
