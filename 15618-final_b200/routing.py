"""Seeded synthetic routing and token rows for the packing workloads.

Stand-in for the reference's data generator (data/gen_synthetic_routing.py):
expert choice follows its Gumbel-max method (gen_zipf_routing, :109-117) --
Gumbel(0, 1) noise per (token, expert), plus the log-prior -s*ln(rank) for a
Zipf popularity p_e ~ 1/rank^s (rank = e + 1, expert 0 hottest), top-K
without replacement.  Unlike the reference (which draws fresh N(0,1) logits
and stores fp16 weights, :120-123), the weights are the fp32 softmax of the K
chosen logits, and token rows are i.i.d. N(0, 1) (the reference uses unit-norm
rows, :51-53), as the workload definitions of this library specify.
"""
from __future__ import annotations

import numpy as np

# Workload definitions (T, d, E, K, distribution, row dtype).
CONFIGS = {
    "c1": dict(T=512, d=2048, E=60, K=4, dist="uniform", dtype="float16", seed=0),
    "c2": dict(T=8192, d=2048, E=60, K=4, dist="zipf", dtype="float16", seed=0),
    "c3": dict(T=65536, d=4096, E=128, K=8, dist="uniform", dtype="bfloat16", seed=0),
    "c4": dict(T=8192, d=2048, E=64, K=4, dist="zipf", dtype="float16", seed=0),
    "c5": dict(T=16384, d=2048, E=60, K=4, dist="zipf", dtype="bfloat16", seed=0, I=1408),
}
ZIPF_S = 1.2


def gen_routing(T: int, K: int, E: int, dist: str = "uniform", seed: int = 0, s: float = ZIPF_S):
    """Returns (assignments int32 [T, K], weights float32 [T, K]).

    Row t lists its K experts in descending score order; weights are the fp32
    softmax of the chosen scores."""
    if K > E:
        raise ValueError(f"K={K} > E={E}")
    rng = np.random.default_rng(seed)
    scores = rng.gumbel(size=(T, E))
    if dist == "zipf":
        scores = scores - s * np.log(np.arange(1, E + 1, dtype=np.float64))[None, :]
    elif dist != "uniform":
        raise ValueError(dist)
    if K < E:
        idx = np.argpartition(-scores, K - 1, axis=1)[:, :K]
    else:
        idx = np.tile(np.arange(E), (T, 1))
    chosen = np.take_along_axis(scores, idx, axis=1)
    order = np.argsort(-chosen, axis=1, kind="stable")
    idx = np.take_along_axis(idx, order, axis=1)
    chosen = np.take_along_axis(chosen, order, axis=1).astype(np.float32)
    z = chosen - chosen.max(axis=1, keepdims=True)
    ez = np.exp(z, dtype=np.float32)
    w = (ez / ez.sum(axis=1, keepdims=True, dtype=np.float32)).astype(np.float32)
    return np.ascontiguousarray(idx.astype(np.int32)), np.ascontiguousarray(w)


def gen_rows(T: int, d: int, dtype: str = "float16", seed: int = 0, device="cpu"):
    """i.i.d. N(0, 1) token rows as a torch tensor of the given 16-bit dtype."""
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(1_000_003 + seed)
    x = torch.randn((T, d), generator=g, device=device, dtype=torch.float32)
    return x.to(getattr(torch, dtype))


def expert_load(asgn: np.ndarray, E: int):
    c = np.bincount(asgn.reshape(-1), minlength=E)
    return c, float(c.max() / c.mean())
