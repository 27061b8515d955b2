"""Regenerate the golden packing vectors in this directory.

Runs the reference's OWN moe::cpu_scatter (src/common/cpu_reference.cpp:12-51,
compiled unchanged into oracle/_ref/libref_cpu.so by `make -C oracle ref`) on
  - the verify.cu mini test (apps/verify.cu:114-128: T=16, K=2, E=4, d=8), and
  - the reference's shipped fixtures results/syn_{uniform,zipf}_T{512,2048,8192}
    (weights converted fp16 -> fp32 as apps/verify.cu:188-196 does; E =
    max(64, max(assignment) + 1) as apps/bench_scatter.cu:154-157 does),
and stores inputs + outputs as compressed .npz.  Embeddings: the T=512
fixtures keep the first 16 columns of the shipped rows (packing is a bitwise
row copy, so a column slice exercises the same row mapping); the larger
fixtures store routing and index outputs only (their outputs do not depend on
the row contents, and the T=8192 rows are not shipped).

Needs the reference tree; run from the repository root:
    make -C oracle ref && python tests/golden/make_golden.py [REFERENCE_DIR]
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import oracle  # noqa: E402


def save(name, **arrays):
    path = os.path.join(HERE, name + ".npz")
    np.savez_compressed(path, **arrays)
    print(f"wrote {path} ({os.path.getsize(path)} bytes)")


def run_ref(emb, asgn, wts, E):
    r = oracle.ref_scatter(emb, asgn, wts, E)
    assert oracle.ref_verify(emb, asgn, wts, r["packed"], r["packed_weights"],
                             r["expert_start"], r["expert_count"], r["perm"], E)
    return r


def mini():
    T, K, E, d = 16, 2, 4, 8
    t = np.arange(T)
    emb = (t[:, None] * 100 + np.arange(d)[None, :]).astype(np.uint16)
    asgn = np.stack([t % E, (t + 1) % E], axis=1).astype(np.int32)
    tf = t.astype(np.float32)
    wts = np.stack([np.float32(0.3) + np.float32(0.001) * tf,
                    np.float32(0.7) - np.float32(0.001) * tf], axis=1).astype(np.float32)
    r = run_ref(emb, asgn, wts, E)
    save("verify_mini", emb=emb, asgn=asgn, wts=wts, E=np.int32(E), packed=r["packed"],
         packed_weights=r["packed_weights"], perm=r["perm"], expert_start=r["expert_start"],
         expert_count=r["expert_count"])


def fixture(ref_dir, prefix, keep_cols):
    res = os.path.join(ref_dir, "results")
    asgn = np.load(os.path.join(res, prefix + "_assignments.npy")).astype(np.int32)
    w16 = np.load(os.path.join(res, prefix + "_weights.npy"))
    wts = w16.astype(np.float32)  # fp16 -> fp32 is exact
    T, K = asgn.shape
    E = max(64, int(asgn.max()) + 1)
    if keep_cols:
        full = np.load(os.path.join(res, prefix + "_embeddings.npy"), mmap_mode="r")
        emb = np.ascontiguousarray(full[:, :keep_cols]).view(np.uint16)
    else:
        emb = np.zeros((T, 8), np.uint16)
    r = run_ref(emb, asgn, wts, E)
    arrays = dict(asgn=asgn, wts=wts, E=np.int32(E), packed_weights=r["packed_weights"],
                  perm=r["perm"], expert_start=r["expert_start"], expert_count=r["expert_count"])
    if keep_cols:
        arrays.update(emb=emb, packed=r["packed"])
    save("fixture_" + prefix, **arrays)


def main():
    ref_dir = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("MOE_REFERENCE_DIR", "")
    if not ref_dir:
        raise SystemExit("give the reference tree as an argument or in MOE_REFERENCE_DIR")
    if not oracle.ref_available():
        sys.exit("oracle/_ref/libref_cpu.so missing: run `make -C oracle ref` first")
    mini()
    for dist in ("uniform", "zipf"):
        fixture(ref_dir, f"syn_{dist}_T512", 16)
        fixture(ref_dir, f"syn_{dist}_T2048", 0)
        fixture(ref_dir, f"syn_{dist}_T8192", 0)


if __name__ == "__main__":
    main()
