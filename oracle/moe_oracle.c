/*
 * moe_oracle.c -- CPU restatement of the MoE token packing / combine / expert
 * FFN path.  TEST INFRASTRUCTURE ONLY: this file is the checker that the CUDA
 * library is compared against.  It is loaded by tests/, by
 * __graft_entry__.smoke() and by bench.py's cpu_baseline leg, and nothing in
 * the product library links or calls it.
 *
 * Parity pinning: oracle_scatter() and oracle_verify() are checked in
 * tests/test_oracle.py against golden vectors produced by the reference's own
 * moe::cpu_scatter (src/common/cpu_reference.cpp:12-51), compiled unchanged
 * from the reference sources into oracle/_ref by oracle/Makefile, on the
 * reference's shipped fixtures (results/syn_{uniform,zipf}_T{512,2048,8192})
 * and on the verify.cu mini test (apps/verify.cu:114-128).
 *
 * oracle_combine(), oracle_swiglu_expert() and oracle_route() have no
 * counterpart in the reference's CPU code (the reference combines only on the
 * GPU with fp32 atomics, apps/bench_e2e.cu:136-152, its FFN has no
 * activation, apps/bench_e2e.cu:289-299, and it routes only on the GPU,
 * apps/bench_e2e.cu:51-130).  The router and combine restatements are
 * pinned instead against golden vectors produced by the reference's own GPU
 * kernels (apps/bench_e2e.cu compiled unchanged into oracle/_ref/libref_gpu.so
 * by oracle/Makefile and run by tests/golden/make_ref_gpu_golden.py;
 * checked in tests/test_ref_gpu_golden.py): the gate logits and the combine
 * at K = 2 (two fp32 atomic adds onto zero commute exactly) bit for bit, the
 * probabilities, assignments and K = 4 combine within stated bounds.  The
 * SwiGLU expert stays "unpinned" (no reference counterpart): it rests on
 * torch fp32 cross-checks.  oracle_plain_expert() restates the reference's
 * activation-free expert and is pinned against outputs of the reference's
 * own GPU layer (run_e2e, apps/bench_e2e.cu:218-329, compiled unchanged into
 * oracle/_ref/libref_gpu.so) in tests/test_ref_gpu_golden.py.
 *
 * All 16-bit payloads are opaque uint16 words; dtype 0 = fp16, 1 = bf16.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------ */
/* IEEE-754 binary16 / bfloat16 <-> binary32 conversions, written from the
 * format definitions (round-to-nearest-even on narrowing).                  */
/* ------------------------------------------------------------------------ */

static inline uint32_t f32_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float bits_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

float oracle_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t man = h & 0x3ffu;
    if (exp == 0x1fu) return bits_f32(sign | 0x7f800000u | (man << 13));  /* inf / nan */
    if (exp == 0) {
        if (man == 0) return bits_f32(sign);
        /* subnormal: value = man * 2^-24, exact in binary32 */
        float v = (float)man * 5.9604644775390625e-08f;
        return sign ? -v : v;
    }
    return bits_f32(sign | ((exp + 112u) << 23) | (man << 13));
}

uint16_t oracle_f32_to_f16(float f) {
    uint32_t u = f32_bits(f);
    uint16_t sign = (uint16_t)((u >> 16) & 0x8000u);
    uint32_t a = u & 0x7fffffffu;
    if (a >= 0x7f800000u) {                           /* inf or nan */
        return (uint16_t)(sign | 0x7c00u | (a > 0x7f800000u ? 0x200u : 0u));
    }
    if (a >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);   /* rounds to >= 65520 -> inf */
    if (a < 0x38800000u) {                            /* below 2^-14: subnormal or zero */
        /* exact scaling to units of 2^-24, then RNE via the FPU */
        float v = bits_f32(a) * 16777216.0f;          /* * 2^24, exact */
        float r = nearbyintf(v);                      /* default mode is RNE */
        return (uint16_t)(sign | (uint16_t)r);        /* r <= 1024 -> may carry into exp */
    }
    uint32_t exp = (a >> 23) - 112u;
    uint32_t man = a & 0x7fffffu;
    uint32_t half = (exp << 10) | (man >> 13);
    uint32_t rem = man & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (half & 1u))) half += 1u;
    return (uint16_t)(sign | half);
}

float oracle_bf16_to_f32(uint16_t h) { return bits_f32((uint32_t)h << 16); }

uint16_t oracle_f32_to_bf16(float f) {
    uint32_t u = f32_bits(f);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);  /* quiet nan */
    uint32_t lsb = (u >> 16) & 1u;
    u += 0x7fffu + lsb;
    return (uint16_t)(u >> 16);
}

static inline float to_f32(uint16_t h, int dtype) {
    return dtype ? oracle_bf16_to_f32(h) : oracle_f16_to_f32(h);
}
static inline uint16_t from_f32(float f, int dtype) {
    return dtype ? oracle_f32_to_bf16(f) : oracle_f32_to_f16(f);
}

void oracle_f32_to_16_array(const float* in, uint16_t* out, int64_t n, int dtype) {
    for (int64_t i = 0; i < n; ++i) out[i] = from_f32(in[i], dtype);
}
void oracle_16_to_f32_array(const uint16_t* in, float* out, int64_t n, int dtype) {
    for (int64_t i = 0; i < n; ++i) out[i] = to_f32(in[i], dtype);
}

/* ------------------------------------------------------------------------ */
/* Pack (scatter).  Follows cpu_scatter, src/common/cpu_reference.cpp:12-51:
 *   count (:21-25) -> exclusive scan (:27-33) -> serial scatter in ascending
 *   (t, k) with a per-expert cursor (:35-50).
 * Extras beyond the reference: expert_start[E] = T*K (the E+1-th entry the
 * reference's callers allocate, apps/verify.cu:70), and slot_pos[t*K+k] = the
 * packed row of slot (t, k) (the inverse of perm, used by the combine).
 * Returns 0, or -1 if an assignment is outside [0, E).                      */
/* ------------------------------------------------------------------------ */
int oracle_scatter(const uint16_t* emb, const int32_t* asgn, const float* wts,
                   int T, int K, int E, int d,
                   uint16_t* packed, float* packed_w,
                   int32_t* expert_start, int32_t* expert_count,
                   int32_t* perm, int32_t* slot_pos) {
    const int64_t TK = (int64_t)T * K;
    for (int64_t i = 0; i < TK; ++i)
        if (asgn[i] < 0 || asgn[i] >= E) return -1;
    memset(expert_count, 0, sizeof(int32_t) * (size_t)E);
    for (int64_t i = 0; i < TK; ++i) expert_count[asgn[i]] += 1;
    int32_t run = 0;
    for (int e = 0; e < E; ++e) { expert_start[e] = run; run += expert_count[e]; }
    if (expert_start) expert_start[E] = run;
    int32_t* cursor = (int32_t*)calloc((size_t)E, sizeof(int32_t));
    for (int t = 0; t < T; ++t) {
        for (int k = 0; k < K; ++k) {
            int64_t slot = (int64_t)t * K + k;
            int e = asgn[slot];
            int32_t pos = expert_start[e] + cursor[e]++;
            if (packed)
                memcpy(packed + (size_t)pos * d, emb + (size_t)t * d, (size_t)d * 2);
            if (packed_w && wts) packed_w[pos] = wts[slot];
            if (perm) perm[pos] = t;
            if (slot_pos) slot_pos[slot] = pos;
        }
    }
    free(cursor);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* Invariant checker.  Restates verify_scatter_outputs,
 * src/common/cpu_reference.cpp:61-178, invariants (a)-(f); returns the number
 * of violations (0 = pass) instead of printing.                             */
/* ------------------------------------------------------------------------ */
int64_t oracle_verify(const uint16_t* emb, const int32_t* asgn, const float* wts,
                      const uint16_t* packed, const float* packed_w,
                      const int32_t* expert_start, const int32_t* expert_count,
                      const int32_t* perm, int T, int K, int E, int d) {
    int64_t errors = 0;
    const int64_t TK = (int64_t)T * K;
    /* (a) contiguous regions that sum to T*K (:73-86) */
    for (int e = 0; e + 1 < E; ++e)
        if (expert_start[e + 1] != expert_start[e] + expert_count[e]) ++errors;
    if ((int64_t)expert_start[E - 1] + expert_count[E - 1] != TK) ++errors;
    /* (b) every packed row equals the embedding row named by perm (:88-103) */
    for (int64_t pos = 0; pos < TK; ++pos) {
        int t = perm[pos];
        if (t < 0 || t >= T) { ++errors; continue; }
        if (packed && memcmp(packed + (size_t)pos * d, emb + (size_t)t * d, (size_t)d * 2)) ++errors;
    }
    /* (c) counts equal a recount (:105-115) */
    int32_t* recount = (int32_t*)calloc((size_t)E, sizeof(int32_t));
    for (int64_t i = 0; i < TK; ++i) {
        if (asgn[i] < 0 || asgn[i] >= E) { ++errors; continue; }
        recount[asgn[i]] += 1;
    }
    for (int e = 0; e < E; ++e) if (recount[e] != expert_count[e]) ++errors;
    free(recount);
    /* (d) every token appears exactly K times (:117-130) */
    int32_t* seen = (int32_t*)calloc((size_t)(T > 0 ? T : 1), sizeof(int32_t));
    for (int64_t pos = 0; pos < TK; ++pos) {
        int t = perm[pos];
        if (t >= 0 && t < T) seen[t] += 1;
    }
    for (int t = 0; t < T; ++t) if (seen[t] != K) ++errors;
    free(seen);
    /* (e) every row of expert e's region owns an unused (t, k) slot routed to
     * e; (f) its weight compares equal to that slot's weight (:132-172) */
    char* used = (char*)calloc((size_t)(TK > 0 ? TK : 1), 1);
    for (int e = 0; e < E; ++e) {
        int32_t lo = expert_start[e], hi = lo + expert_count[e];
        if (lo < 0 || hi > TK) { ++errors; continue; }
        for (int32_t pos = lo; pos < hi; ++pos) {
            int t = perm[pos];
            if (t < 0 || t >= T) continue;
            int mk = -1;
            for (int k = 0; k < K; ++k) {
                int64_t s = (int64_t)t * K + k;
                if (asgn[s] == e && !used[s]) { used[s] = 1; mk = k; break; }
            }
            if (mk < 0) { ++errors; continue; }
            if (wts && packed_w) {
                if (wts[(int64_t)t * K + mk] != packed_w[pos]) ++errors;
            }
        }
    }
    free(used);
    return errors;
}

/* ------------------------------------------------------------------------ */
/* Weighted unpermute + combine.  Follows the math of unpack_combine_kernel +
 * f32_to_f16_kernel (apps/bench_e2e.cu:136-152): out[t] = round16( sum over
 * the K packed rows of token t of w * f32(y[pos]) ), accumulated in fp32.
 * The reference sums with order-dependent atomics; here the sum runs in
 * ascending k with one fused multiply-add per term, the order the CUDA
 * kernel uses, so results are comparable bit for bit.                      */
/* ------------------------------------------------------------------------ */
static float g_f16_lut[65536];

__attribute__((constructor)) static void init_f16_lut(void) {
    for (uint32_t i = 0; i < 65536u; ++i) g_f16_lut[i] = oracle_f16_to_f32((uint16_t)i);
}

/* Built twice (FMA hardware and generic); the loader picks the one the host
 * supports.  Both compute the same correctly rounded fmaf.                  */
__attribute__((target_clones("fma", "default")))
void oracle_combine(const uint16_t* y, const float* packed_w, const int32_t* slot_pos,
                    int T, int K, int d, int dtype, uint16_t* out) {
    float* acc = (float*)malloc(sizeof(float) * (size_t)(d > 0 ? d : 1));
    for (int t = 0; t < T; ++t) {
        for (int i = 0; i < d; ++i) acc[i] = 0.0f;
        for (int k = 0; k < K; ++k) {
            int32_t pos = slot_pos[(int64_t)t * K + k];
            float w = packed_w[pos];
            const uint16_t* row = y + (size_t)pos * d;
            if (dtype)
                for (int i = 0; i < d; ++i) acc[i] = fmaf(w, bits_f32((uint32_t)row[i] << 16), acc[i]);
            else
                for (int i = 0; i < d; ++i) acc[i] = fmaf(w, g_f16_lut[row[i]], acc[i]);
        }
        for (int i = 0; i < d; ++i) out[(size_t)t * d + i] = from_f32(acc[i], dtype);
    }
    free(acc);
}

/* Reference-order variant (apps/bench_e2e.cu:136-147): walks packed rows in
 * ascending pos and accumulates into an fp32 [T, d] buffer via perm; used to
 * check that the reference's own formulation agrees within tolerance.       */
void oracle_combine_by_perm(const uint16_t* y, const float* packed_w, const int32_t* perm,
                            int TK, int T, int d, int dtype, float* out32) {
    memset(out32, 0, sizeof(float) * (size_t)T * (size_t)d);
    for (int pos = 0; pos < TK; ++pos) {
        int t = perm[pos];
        float w = packed_w[pos];
        for (int i = 0; i < d; ++i)
            out32[(size_t)t * d + i] += w * to_f32(y[(size_t)pos * d + i], dtype);
    }
}

/* ------------------------------------------------------------------------ */
/* One SwiGLU expert on M rows, fp32 accumulate.  No reference counterpart
 * (the reference FFN is up*down with no activation, apps/bench_e2e.cu:289-299).
 *   x     [M, D]      rows (dtype)
 *   w_gu  [2*I, D]    row j < I is the gate column j, row I + j the up column j
 *   w_dn  [D, I]      row n is output column n over the I inner features
 *   h     = silu(x . gate) * (x . up)  rounded to dtype (the materialised
 *           intermediate), y = h . down rounded to dtype.                   */
/* ------------------------------------------------------------------------ */
void oracle_swiglu_expert(const uint16_t* x, const uint16_t* w_gu, const uint16_t* w_dn,
                          int M, int D, int I, int dtype, uint16_t* h_out, uint16_t* y_out) {
    float* xf = (float*)malloc(sizeof(float) * (size_t)D);
    float* hf = (float*)malloc(sizeof(float) * (size_t)I);
    float* wrow = (float*)malloc(sizeof(float) * (size_t)(D > I ? D : I));
    float* gacc = (float*)malloc(sizeof(float) * (size_t)I);
    float* uacc = (float*)malloc(sizeof(float) * (size_t)I);
    for (int m = 0; m < M; ++m) {
        for (int c = 0; c < D; ++c) xf[c] = to_f32(x[(size_t)m * D + c], dtype);
        for (int j = 0; j < I; ++j) {
            double g = 0.0, u = 0.0;
            const uint16_t* gr = w_gu + (size_t)j * D;
            const uint16_t* ur = w_gu + (size_t)(I + j) * D;
            for (int c = 0; c < D; ++c) {
                g += (double)xf[c] * to_f32(gr[c], dtype);
                u += (double)xf[c] * to_f32(ur[c], dtype);
            }
            gacc[j] = (float)g; uacc[j] = (float)u;
        }
        for (int j = 0; j < I; ++j) {
            float g = gacc[j];
            float s = g / (1.0f + expf(-g));
            uint16_t hb = from_f32(s * uacc[j], dtype);
            if (h_out) h_out[(size_t)m * I + j] = hb;
            hf[j] = to_f32(hb, dtype);
        }
        for (int n = 0; n < D; ++n) {
            const uint16_t* dr = w_dn + (size_t)n * I;
            double acc = 0.0;
            for (int j = 0; j < I; ++j) acc += (double)hf[j] * to_f32(dr[j], dtype);
            y_out[(size_t)m * D + n] = from_f32((float)acc, dtype);
        }
    }
    free(xf); free(hf); free(wrow); free(gacc); free(uacc);
}

/* One activation-free expert on M rows: the reference's FFN (per-expert
 * cublasHgemm up then down, apps/bench_e2e.cu:274-301) restated with fp32
 * products summed in double, each result rounded once to dtype.
 *   x     [M, D]      rows (dtype)
 *   w_up  [F, D]      row j = inner feature j (the reference's W1[e] transposed)
 *   w_dn  [D, F]      row n = output column n (the reference's W2[e] transposed)
 *   mid   = x . w_up^T rounded to dtype, y = mid . w_dn^T rounded to dtype.
 * Pinned against the reference's own GPU layer (tests/test_ref_gpu_golden.py). */
void oracle_plain_expert(const uint16_t* x, const uint16_t* w_up, const uint16_t* w_dn, int M, int D, int F,
                         int dtype, uint16_t* mid_out, uint16_t* y_out) {
    float* xf = (float*)malloc(sizeof(float) * (size_t)D);
    float* mf = (float*)malloc(sizeof(float) * (size_t)F);
    for (int m = 0; m < M; ++m) {
        for (int c = 0; c < D; ++c) xf[c] = to_f32(x[(size_t)m * D + c], dtype);
        for (int j = 0; j < F; ++j) {
            const uint16_t* ur = w_up + (size_t)j * D;
            double acc = 0.0;
            for (int c = 0; c < D; ++c) acc += (double)xf[c] * to_f32(ur[c], dtype);
            const uint16_t mb = from_f32((float)acc, dtype);
            if (mid_out) mid_out[(size_t)m * F + j] = mb;
            mf[j] = to_f32(mb, dtype);
        }
        for (int n = 0; n < D; ++n) {
            const uint16_t* dr = w_dn + (size_t)n * F;
            double acc = 0.0;
            for (int j = 0; j < F; ++j) acc += (double)mf[j] * to_f32(dr[j], dtype);
            y_out[(size_t)m * D + n] = from_f32((float)acc, dtype);
        }
    }
    free(xf); free(mf);
}

/* ------------------------------------------------------------------------ */
/* The reference's deterministic input fills (include/moe/fp16_host.hpp:22-39):
 * a 32-bit linear congruential generator s <- s * 1664525 + 1013904223, value
 * ((s >> 16) / 65536 - 0.5) * 2 * half_range in float, rounded to fp16
 * (round-to-nearest-even, as __float2half) for the half fill.  Used to
 * regenerate the inputs of golden vectors made by the reference's GPU code. */
/* ------------------------------------------------------------------------ */
static inline float lcg_value(uint32_t* s, float half_range) {
    *s = *s * 1664525u + 1013904223u;
    float x = (float)(*s >> 16) / 65536.0f - 0.5f;
    return x * 2.0f * half_range;
}

void oracle_fill_random_half(uint16_t* buf, int64_t n, uint32_t seed, float half_range) {
    uint32_t s = seed;
    for (int64_t i = 0; i < n; ++i) buf[i] = oracle_f32_to_f16(lcg_value(&s, half_range));
}

void oracle_fill_random_float(float* buf, int64_t n, uint32_t seed, float half_range) {
    uint32_t s = seed;
    for (int64_t i = 0; i < n; ++i) buf[i] = lcg_value(&s, half_range);
}

/* Gate logits alone, [T, E] fp32: gate_kernel (apps/bench_e2e.cu:52-62) and
 * the first loop of fused_route_kernel (:101-102), i.e. one float fused
 * multiply-add per input feature in ascending i (nvcc contracts the
 * reference's `acc += a * b`).                                              */
__attribute__((target_clones("fma", "default")))
void oracle_gate_logits(const uint16_t* emb, const float* w_gate, int T, int d, int E, int dtype,
                        float* logits) {
    for (int t = 0; t < T; ++t)
        for (int e = 0; e < E; ++e) {
            float acc = 0.f;
            for (int i = 0; i < d; ++i)
                acc = fmaf(to_f32(emb[(size_t)t * d + i], dtype), w_gate[(size_t)i * E + e], acc);
            logits[(size_t)t * E + e] = acc;
        }
}

/* ------------------------------------------------------------------------ */
/* Router: gate GEMM + softmax over all E + top-K (apps/bench_e2e.cu:95-130,
 * fused_route_kernel; the unfused gate/softmax/topk kernels :51-93 compute
 * the same).  emb [T, d] 16-bit, w_gate [d, E] fp32 (row i = input feature).
 *   mode 0: the reference's own arithmetic -- logit accumulated in float in
 *           ascending i as fmaf(x_i, W[i*E+e], logit) (nvcc contracts the
 *           reference's `logit += a * b` into a fused multiply-add), max,
 *           expf(l - max) summed in ascending e, one division per expert,
 *           K rounds of strict-greater argmax (ties to the lower index);
 *   mode 1: logits and softmax in double, the order-independent target;
 *           weights rounded to float at the end.
 * margin[t] (may be NULL): p_K - p_{K+1} of the double computation (1 when
 * K == E); a token with a tiny margin may legitimately select a different
 * K-th expert under another summation order.                               */
void oracle_route(const uint16_t* emb, const float* w_gate, int T, int d, int E, int K, int dtype, int mode,
                  int32_t* asgn, float* wts, double* margin) {
    float* x = (float*)malloc(sizeof(float) * (size_t)d);
    float* pf = (float*)malloc(sizeof(float) * (size_t)E);
    double* pd = (double*)malloc(sizeof(double) * (size_t)E);
    for (int t = 0; t < T; ++t) {
        for (int i = 0; i < d; ++i) x[i] = to_f32(emb[(size_t)t * d + i], dtype);
        for (int e = 0; e < E; ++e) {
            double ld = 0.0;
            float lf = 0.f;
            for (int i = 0; i < d; ++i) {
                const float w = w_gate[(size_t)i * E + e];
                ld += (double)x[i] * (double)w;
                lf = fmaf(x[i], w, lf);
            }
            pd[e] = ld;
            pf[e] = lf;
        }
        /* double softmax (also gives the margin) */
        double mxd = pd[0];
        for (int e = 1; e < E; ++e) if (pd[e] > mxd) mxd = pd[e];
        double sd = 0.0;
        for (int e = 0; e < E; ++e) { pd[e] = exp(pd[e] - mxd); sd += pd[e]; }
        for (int e = 0; e < E; ++e) pd[e] /= sd;
        /* float softmax, the reference's sequence */
        float mxf = pf[0];
        for (int e = 1; e < E; ++e) mxf = fmaxf(mxf, pf[e]);
        float sf = 0.f;
        for (int e = 0; e < E; ++e) { pf[e] = expf(pf[e] - mxf); sf += pf[e]; }
        for (int e = 0; e < E; ++e) pf[e] /= sf;
        double kth = 0.0;
        for (int k = 0; k < K; ++k) {
            int best = 0;
            if (mode == 0) {
                for (int e = 1; e < E; ++e) if (pf[e] > pf[best]) best = e;
                asgn[(size_t)t * K + k] = best;
                wts[(size_t)t * K + k] = pf[best];
                pf[best] = -1.f;
            } else {
                for (int e = 1; e < E; ++e) if (pd[e] > pd[best]) best = e;
                asgn[(size_t)t * K + k] = best;
                wts[(size_t)t * K + k] = (float)pd[best];
            }
            if (mode != 0) { kth = pd[best]; pd[best] = -1.0; }
        }
        if (margin) {
            if (mode == 0) {  /* recompute the double ranking for the margin */
                double p1 = -1.0, p2 = -1.0;  /* K-th and (K+1)-th largest */
                for (int k = 0; k <= K && k < E; ++k) {
                    int best = 0;
                    for (int e = 1; e < E; ++e) if (pd[e] > pd[best]) best = e;
                    if (k == K - 1) p1 = pd[best];
                    if (k == K) p2 = pd[best];
                    pd[best] = -1.0;
                }
                margin[t] = K >= E ? 1.0 : p1 - p2;
            } else {
                double nxt = -1.0;
                for (int e = 0; e < E; ++e) if (pd[e] > nxt) nxt = pd[e];
                margin[t] = K >= E ? 1.0 : kth - nxt;
            }
        }
    }
    free(x); free(pf); free(pd);
}
