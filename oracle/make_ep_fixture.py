"""Input files for the reference's own expert-parallel harness
(apps/bench_prefill.cu, compiled unchanged into oracle/_ref/bench_prefill_b200
by `make -C oracle ref-apps`), built from the same seeded batches that
bench.py feeds this library, so the two runs see identical tokens.

TEST / COMPARATOR INFRASTRUCTURE: nothing in the library uses it.

bench_prefill reads <dir>/<prefix>_{embeddings,assignments,weights}.npy
(apps/bench_prefill.cu:326-328): embeddings fp16 [T_full, d], assignments int32
[rounds * T_full, K], weights fp32 [rounds * T_full, K], and gives rank r the
rows [r * T_full / N, (r + 1) * T_full / N) (:341-395).  Here T_full = N * T and
rank r's slice is exactly bench.py's rank-r batch of the config (seed + r), so
config c4 (T = 8192 per GPU, d = 2048, E = 64, K = 4) lines up with
`bench.py --gpus N --config c4 --placement contiguous --replicate 0`.

  python oracle/make_ep_fixture.py OUT_DIR PREFIX N [c4|c4u]
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "15618-final_b200"))
import routing  # noqa: E402


def main(out_dir, prefix, n, cfg="c4"):
    import torch
    c = dict(routing.CONFIGS["c4"])
    if cfg == "c4u":
        c["dist"] = "uniform"
    T, d, E, K = c["T"], c["d"], c["E"], c["K"]
    embs, asgns, wtss = [], [], []
    for r in range(n):
        a, w = routing.gen_routing(T, K, E, c["dist"], c["seed"] + r)
        x = routing.gen_rows(T, d, c["dtype"], c["seed"] + r)
        embs.append(x.view(torch.int16).numpy().view(np.float16))
        asgns.append(a)
        wtss.append(w)
    os.makedirs(out_dir, exist_ok=True)
    np.save(os.path.join(out_dir, f"{prefix}_embeddings.npy"), np.concatenate(embs))
    np.save(os.path.join(out_dir, f"{prefix}_assignments.npy"), np.concatenate(asgns).astype(np.int32))
    np.save(os.path.join(out_dir, f"{prefix}_weights.npy"), np.concatenate(wtss).astype(np.float32))
    print(f"wrote {prefix}: T_full={n * T} d={d} E={E} K={K} {c['dist']}")


if __name__ == "__main__":
    main(sys.argv[1], sys.argv[2], int(sys.argv[3]), sys.argv[4] if len(sys.argv) > 4 else "c4")
