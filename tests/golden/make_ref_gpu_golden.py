"""Generate the golden vectors of the reference's own GPU router, combine and
whole MoE layer (router -> IScatter -> per-expert cublasHgemm FFN -> combine).

The reference has no CPU router or combine: it routes and combines only on the
GPU, in kernels local to apps/bench_e2e.cu (gate_kernel / softmax_kernel /
topk_kernel :52-93, fused_route_kernel :95-130, unpack_combine_kernel +
f32_to_f16_kernel :136-152).  `make -C oracle ref-gpu` compiles that file
unchanged into oracle/_ref/libref_gpu.so behind C launchers that use the
reference's launch shapes; this script runs them on inputs made by the
reference's own deterministic fills (include/moe/fp16_host.hpp:22-39) and
stores the outputs as ref_gpu_{route,combine,layer}_<case>.npz.  Inputs are not
stored: the tests regenerate them with the oracle's restatement of the fills
(checked against the `*_sum` checksums below, which come from the reference's
own fill functions).

Needs a CUDA GPU and the reference-built library; run from the repository
root:  make -C oracle ref-gpu && python tests/golden/make_ref_gpu_golden.py [OUT_DIR [layer]]
"""
import ctypes
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import oracle  # noqa: E402

P, I = ctypes.c_void_p, ctypes.c_int

# name, T, d, E, K, emb seed, emb half-range, gate seed, gate half-range
ROUTE_CASES = [
    ("mini", 16, 8, 4, 2, 1, 0.01, 2, 0.05),         # bench_e2e.cu:331-343 mini-test inputs
    ("flat_e60", 256, 512, 60, 4, 11, 0.01, 12, 0.05),  # the fills' default ranges
    ("sharp_e60", 256, 2048, 60, 4, 21, 1.0, 22, 0.05),
    ("e128_k8", 128, 1024, 128, 8, 31, 1.0, 32, 0.05),
    ("e8_k2", 64, 256, 8, 2, 41, 1.0, 42, 0.05),
]

# name, T, K, E, d, expert-output seed, half-range, weight seed
COMBINE_CASES = [
    ("k2", 128, 2, 60, 256, 51, 1.0, 52),   # two atomic adds onto zero: order-free
    ("k4", 64, 4, 60, 256, 61, 1.0, 62),    # four: order-dependent on the GPU
]


# The reference's whole layer (run_e2e, apps/bench_e2e.cu:218-329): router,
# IScatter "sort", per-expert cublasHgemm up/down (no activation), combine.
# name, T, K, E, d, F, zipf prior, emb seed, gate seed, gate half-range, w1 seed, w2 seed
LAYER_CASES = [
    ("flat", 256, 2, 8, 128, 512, False, 71, 72, 0.05, 73, 74),   # near-uniform routing, d_ffn = 4d
    ("zipf", 512, 4, 16, 64, 256, True, 81, 82, 0.5, 83, 84),     # skewed segments, d_ffn = 4d
]
MID_EVERY = 8       # mid rows stored: every 8th packed row (plus every row's sum of squares)


def layer_inputs(fill_half, fill_float, T, K, E, d, F, zipf, es, gs, gr, w1s, w2s):
    """Inputs of a layer case from the reference's fills (the tests rebuild
    them with the oracle's restatement of the same fills).  Rows in [-1, 1),
    expert weights in [-2/sqrt(K_dim), 2/sqrt(K_dim)) so every product is O(1).
    Zipf cases: feature 0 of every token is 1.0 and gate row 0 carries the
    log-prior -1.2 ln(e + 1), so the reference's router picks skewed experts."""
    emb = fill_half(T * d, es, 1.0).reshape(T, d)
    wg = fill_float(d * E, gs, gr).reshape(d, E)
    if zipf:
        emb[:, 0] = 0x3C00
        wg[0, :] += (-1.2 * np.log(np.arange(1, E + 1))).astype(np.float32)
    w1 = fill_half(E * d * F, w1s, 2.0 / np.sqrt(d)).reshape(E, d, F)
    w2 = fill_half(E * F * d, w2s, 2.0 / np.sqrt(F)).reshape(E, F, d)
    return np.ascontiguousarray(emb), np.ascontiguousarray(wg), w1, w2


def lib():
    so = os.path.join(ROOT, "oracle", "_ref", "libref_gpu.so")
    L = ctypes.CDLL(so)
    L.ref_fill_random_half.argtypes = [P, ctypes.c_size_t, ctypes.c_uint32, ctypes.c_float]
    L.ref_fill_random_half.restype = None
    L.ref_fill_random_float.argtypes = [P, ctypes.c_size_t, ctypes.c_uint32, ctypes.c_float]
    L.ref_fill_random_float.restype = None
    L.ref_gpu_fused_route.argtypes = [P, P, I, I, I, I, P, P]
    L.ref_gpu_fused_route.restype = I
    L.ref_gpu_naive_route.argtypes = [P, P, I, I, I, I, P, P, P, P]
    L.ref_gpu_naive_route.restype = I
    L.ref_gpu_unpack_combine.argtypes = [P, P, P, I, I, I, P, P]
    L.ref_gpu_unpack_combine.restype = I
    L.ref_gpu_moe_layer.argtypes = [P, P, P, P, I, I, I, I, I, ctypes.c_char_p, I] + [P] * 9
    L.ref_gpu_moe_layer.restype = I
    return L


def ptr(a):
    return a.ctypes.data_as(P)


def ref_half(L, n, seed, hr):
    out = np.empty(n, np.uint16)
    L.ref_fill_random_half(ptr(out), n, seed, hr)
    return out


def ref_float(L, n, seed, hr):
    out = np.empty(n, np.float32)
    L.ref_fill_random_float(ptr(out), n, seed, hr)
    return out


def combine_layout(T, K, E):
    """A packed layout for the combine: slot (t, k) goes to expert
    (7t + 13k) mod E (distinct over k for K <= 4), packed by the oracle's
    cpu_scatter restatement.  Returns perm [TK] and the (t, k) of each row."""
    t = np.arange(T)[:, None]
    k = np.arange(K)[None, :]
    asgn = ((7 * t + 13 * k) % E).astype(np.int32)
    wts = np.zeros((T, K), np.float32)
    r = oracle.scatter(np.zeros((T, 1), np.uint16), asgn, wts, E)
    return r["perm"]


def main(out_dir, only=None):
    os.makedirs(out_dir, exist_ok=True)
    L = lib()

    def save(name, **arrays):
        path = os.path.join(out_dir, name + ".npz")
        np.savez_compressed(path, **arrays)
        print(f"wrote {path} ({os.path.getsize(path)} bytes)")

    if only == "layer":
        make_layer_goldens(L, save)
        return

    for name, T, d, E, K, es, er, gs, gr in ROUTE_CASES:
        emb = ref_half(L, T * d, es, er)
        wg = ref_float(L, d * E, gs, gr)
        fa = np.empty(T * K, np.int32)
        fw = np.empty(T * K, np.float32)
        rc = L.ref_gpu_fused_route(ptr(emb), ptr(wg), T, K, E, d, ptr(fa), ptr(fw))
        assert rc == 0, f"fused_route_kernel: cuda error {rc}"
        lg = np.empty(T * E, np.float32)
        pr = np.empty(T * E, np.float32)
        na = np.empty(T * K, np.int32)
        nw = np.empty(T * K, np.float32)
        rc = L.ref_gpu_naive_route(ptr(emb), ptr(wg), T, K, E, d, ptr(lg), ptr(pr), ptr(na), ptr(nw))
        assert rc == 0, f"gate/softmax/topk kernels: cuda error {rc}"
        save(f"ref_gpu_route_{name}",
             T=np.int32(T), d=np.int32(d), E=np.int32(E), K=np.int32(K),
             emb_seed=np.uint32(es), emb_range=np.float32(er),
             gate_seed=np.uint32(gs), gate_range=np.float32(gr),
             emb_sum=np.int64(emb.astype(np.int64).sum()),
             gate_sum=np.int64(wg.view(np.uint32).astype(np.int64).sum()),
             fused_asgn=fa.reshape(T, K), fused_wts=fw.reshape(T, K),
             logits=lg.reshape(T, E), probs=pr.reshape(T, E),
             naive_asgn=na.reshape(T, K), naive_wts=nw.reshape(T, K))

    for name, T, K, E, d, ys, yr, ws in COMBINE_CASES:
        TK = T * K
        perm = combine_layout(T, K, E)
        y = ref_half(L, TK * d, ys, yr)
        pw = ref_float(L, TK, ws, 0.5)
        o32 = np.empty(T * d, np.float32)
        o16 = np.empty(T * d, np.uint16)
        rc = L.ref_gpu_unpack_combine(ptr(y), ptr(pw), ptr(perm), TK, T, d, ptr(o32), ptr(o16))
        assert rc == 0, f"unpack_combine_kernel: cuda error {rc}"
        save(f"ref_gpu_combine_{name}",
             T=np.int32(T), K=np.int32(K), E=np.int32(E), d=np.int32(d),
             y_seed=np.uint32(ys), y_range=np.float32(yr), w_seed=np.uint32(ws),
             w_range=np.float32(0.5), y_sum=np.int64(y.astype(np.int64).sum()),
             perm=perm, packed_weights=pw, out32=o32.reshape(T, d), out16=o16.reshape(T, d))

    make_layer_goldens(L, save)


def make_layer_goldens(L, save):
    for name, T, K, E, d, F, zipf, es, gs, gr, w1s, w2s in LAYER_CASES:
        emb, wg, w1, w2 = layer_inputs(lambda n, sd, hr: ref_half(L, n, sd, hr),
                                       lambda n, sd, hr: ref_float(L, n, sd, hr),
                                       T, K, E, d, F, zipf, es, gs, gr, w1s, w2s)
        TK = T * K
        a = np.empty(TK, np.int32)
        rw = np.empty(TK, np.float32)
        perm = np.empty(TK, np.int32)
        pw = np.empty(TK, np.float32)
        st = np.empty(E, np.int32)
        ct = np.empty(E, np.int32)
        mid = np.empty(TK * F, np.uint16)
        y = np.empty(TK * d, np.uint16)
        out = np.empty(T * d, np.uint16)
        rc = L.ref_gpu_moe_layer(ptr(emb), ptr(wg), ptr(w1), ptr(w2), T, K, E, d, F, b"sort", 1, ptr(a), ptr(rw),
                                 ptr(perm), ptr(pw), ptr(st), ptr(ct), ptr(mid), ptr(y), ptr(out))
        assert rc == 0, f"run_e2e: cuda error {rc}"
        mid = mid.reshape(TK, F)
        mid32 = oracle.to_f32(mid, 0).astype(np.float64)
        save(f"ref_gpu_layer_{name}",
             T=np.int32(T), K=np.int32(K), E=np.int32(E), d=np.int32(d), F=np.int32(F), zipf=np.int32(zipf),
             emb_seed=np.uint32(es), gate_seed=np.uint32(gs), gate_range=np.float32(gr),
             w1_seed=np.uint32(w1s), w2_seed=np.uint32(w2s),
             emb_sum=np.int64(emb.astype(np.int64).sum()),
             w1_sum=np.int64(w1.astype(np.int64).sum()), w2_sum=np.int64(w2.astype(np.int64).sum()),
             asgn=a.reshape(T, K), rwt=rw.reshape(T, K), perm=perm, packed_weights=pw,
             expert_start=st, expert_count=ct, mid_every=np.int32(MID_EVERY), mid_rows=mid[::MID_EVERY],
             mid_sumsq=(mid32 * mid32).sum(axis=1), y=y.reshape(TK, d), out=out.reshape(T, d))


if __name__ == "__main__":
    # [OUT_DIR [layer]]: "layer" makes the layer goldens only
    main(sys.argv[1] if len(sys.argv) > 1 else HERE, sys.argv[2] if len(sys.argv) > 2 else None)
