"""The CUDA router (moe_b200_route) and combine (moe_b200_unpermute) against
the outputs of the reference's OWN GPU kernels (fused_route_kernel,
unpack_combine_kernel + f32_to_f16_kernel, apps/bench_e2e.cu:95-152), stored
in tests/golden/ref_gpu_*.npz by tests/golden/make_ref_gpu_golden.py.

Bounds (the same as the oracle-based GPU tests):
  - router: assignments identical for every token whose reference top-(K+1)
    probabilities are at least MARGIN apart (relative, consecutive); routing
    weights within RTOL relative on the tokens whose assignments agree (the
    tensor cores accumulate each logit in a different fp32 order than the
    reference's sequential sum);
  - combine: within one fp16 ulp of the reference's output (the reference
    multiplies, then adds atomically; the kernel fuses each term into one
    FMA), and bit for bit equal to the oracle's product-order restatement.
"""
import glob
import os

import numpy as np
import pytest
import torch

import moe_b200 as mb
import oracle

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
ROUTE = sorted(glob.glob(os.path.join(GOLDEN, "ref_gpu_route_*.npz")))
COMBINE = sorted(glob.glob(os.path.join(GOLDEN, "ref_gpu_combine_*.npz")))
MARGIN = 5e-4
RTOL = 1e-4


def _name(p):
    return os.path.basename(p)[len("ref_gpu_"):-len(".npz")]


def _dev16(u16):
    return torch.from_numpy(np.ascontiguousarray(u16).view(np.int16)).cuda().view(torch.float16)


@pytest.mark.parametrize("path", ROUTE, ids=_name)
def test_route_kernel_vs_reference_gpu(cuda, path):
    g = np.load(path)
    T, d, E, K = (int(g[k]) for k in ("T", "d", "E", "K"))
    emb = oracle.fill_random_half(T * d, int(g["emb_seed"]), float(g["emb_range"])).reshape(T, d)
    wg = oracle.fill_random_float(d * E, int(g["gate_seed"]), float(g["gate_range"])).reshape(d, E)
    rw = mb.RouterWeights(torch.from_numpy(wg).cuda(), torch.float16)
    a, p = mb.route(_dev16(emb), rw, K)
    torch.cuda.synchronize()
    assert mb.device_status() == 0
    a, p = a.cpu().numpy(), p.cpu().numpy()
    ra, rp = g["fused_asgn"], g["fused_wts"]
    top = -np.sort(-g["probs"], axis=1)[:, :K + 1]
    sep = ((top[:, :-1] - top[:, 1:]) / top[:, :-1]).min(axis=1) >= MARGIN
    assert np.array_equal(a[sep], ra[sep])
    same = (a == ra).all(axis=1)
    assert same.mean() > 0.9
    np.testing.assert_allclose(p[same], rp[same], rtol=RTOL, atol=0)


@pytest.mark.parametrize("path", COMBINE, ids=_name)
def test_unpermute_kernel_vs_reference_gpu(cuda, path):
    g = np.load(path)
    T, K, E, d = (int(g[k]) for k in ("T", "K", "E", "d"))
    y = oracle.fill_random_half(T * K * d, int(g["y_seed"]), float(g["y_range"])).reshape(T * K, d)
    pw = g["packed_weights"]
    t = np.arange(T)[:, None]
    k = np.arange(K)[None, :]
    asgn = ((7 * t + 13 * k) % E).astype(np.int32)
    r = oracle.scatter(np.zeros((T, 1), np.uint16), asgn, np.zeros((T, K), np.float32), E)
    assert np.array_equal(r["perm"], g["perm"])
    out = mb.unpermute(_dev16(y), torch.from_numpy(pw).cuda(), torch.from_numpy(r["slot_pos"]).cuda(), T, K)
    torch.cuda.synchronize()
    assert mb.device_status() == 0
    got = out.view(torch.int16).cpu().numpy().view(np.uint16)
    assert np.abs(got.astype(np.int32) - g["out16"].astype(np.int32)).max() <= 1
    assert got.tobytes() == oracle.combine(y, pw, r["slot_pos"], T, K, 0).tobytes()
