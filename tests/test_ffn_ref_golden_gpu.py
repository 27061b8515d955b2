"""The activation-free grouped FFN (moe_b200_grouped_ffn) and the whole
pack -> FFN -> unpermute path against the reference's OWN single-GPU layer
(run_e2e, apps/bench_e2e.cu:218-329: fused router, IScatter "sort",
per-expert cublasHgemm up/down with no activation, atomic combine), whose
outputs tests/golden/make_ref_gpu_golden.py stored in
tests/golden/ref_gpu_layer_<case>.npz.

The reference's routing (its assignments and weights) is fed to this
library's pack, so the comparison isolates the packing, the FFN and the
combine:
  - pack: perm / expert_start / expert_count / packed weights bit for bit;
  - weight conversion (moe_b200_ffn_weights_from_reference): an exact
    transpose;
  - FFN: every element of mid and y within FFN_ABS absolute or FFN_REL
    relative of the reference's cublasHgemm output (ten times tighter in
    absolute terms than the reference's own GEMM check,
    apps/grouped_gemm_test.cu:253-269), and within 2e-3 (mid) / 4e-3 (y)
    absolute plus relative of the oracle's restatement;
  - output: the combine bit-exact on this library's expert outputs, and
    the layer output within the FFN bound of the reference layer's output.
"""
import glob
import os

import numpy as np
import pytest
import torch

import moe_b200 as mb
import oracle
from test_ref_gpu_golden import FFN_ABS, FFN_REL, ffn_close, layer_inputs, oracle_layer_ffn

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
LAYER = sorted(glob.glob(os.path.join(GOLDEN, "ref_gpu_layer_*.npz")))


def _name(p):
    return os.path.basename(p)[len("ref_gpu_"):-len(".npz")]


def _dev16(u16):
    return torch.from_numpy(np.ascontiguousarray(u16).view(np.int16)).cuda().view(torch.float16)


def _host16(t):
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


@pytest.mark.parametrize("path", LAYER, ids=_name)
def test_grouped_ffn_vs_reference_layer(cuda, path):
    g = np.load(path)
    T, K, E, d, F = (int(g[k]) for k in ("T", "K", "E", "d", "F"))
    emb, _, w1, w2 = layer_inputs(g)
    x = _dev16(emb)
    a = torch.from_numpy(np.ascontiguousarray(g["asgn"])).cuda()
    w = torch.from_numpy(np.ascontiguousarray(g["rwt"])).cuda()
    r = mb.pack(x, a, w, E)
    w_up, w_down = mb.ffn_weights_from_reference(_dev16(w1), _dev16(w2))
    mid, y = mb.grouped_ffn(r.packed, r.expert_start, w_up, w_down)
    out = mb.unpermute(y, r.packed_weights, r.slot_pos, T, K)
    torch.cuda.synchronize()
    assert mb.device_status() == 0

    # packing: the reference strategy's order, bit for bit
    assert np.array_equal(r.perm.cpu().numpy(), g["perm"])
    assert np.array_equal(r.expert_start.cpu().numpy()[:E], g["expert_start"])
    assert np.array_equal(r.expert_count.cpu().numpy(), g["expert_count"])
    assert np.array_equal(r.packed_weights.cpu().numpy().view(np.uint32), g["packed_weights"].view(np.uint32))
    # weight conversion: an exact transpose
    assert np.array_equal(_host16(w_up), np.ascontiguousarray(w1.transpose(0, 2, 1)))
    assert np.array_equal(_host16(w_down), np.ascontiguousarray(w2.transpose(0, 2, 1)))

    mid_h, y_h, out_h = _host16(mid), _host16(y), _host16(out)
    every = int(g["mid_every"])
    ok, da, dr = ffn_close(mid_h[::every], g["mid_rows"])
    assert ok, ("mid vs reference", da, dr, FFN_ABS, FFN_REL)
    ok, da, dr = ffn_close(y_h, g["y"])
    assert ok, ("y vs reference", da, dr, FFN_ABS, FFN_REL)
    # the restatement: fp32 tensor-core accumulation vs a double sum, one
    # 16-bit rounding each
    o_mid, o_y = oracle_layer_ffn(g, emb, w1, w2)
    for got, want, tol in ((mid_h, o_mid, 2e-3), (y_h, o_y, 4e-3)):
        w32 = oracle.to_f32(want, 0).astype(np.float64)
        err = np.abs(oracle.to_f32(got, 0) - w32)
        assert (err <= tol + tol * np.abs(w32)).all(), err.max()
    # the layer's output: the combine is bit-exact on this library's expert
    # outputs, and within the FFN bound of the reference layer's output (its
    # terms carry the FFN's rounding differences; cancellation between the K
    # terms rules out an ulp bound)
    assert out_h.tobytes() == oracle.combine(y_h, g["packed_weights"], r.slot_pos.cpu().numpy(), T, K, 0).tobytes()
    ok, da, dr = ffn_close(out_h, g["out"])
    assert ok, ("output vs reference", da, dr)


@pytest.mark.parametrize("F", [16, 272])   # one partial N block / several K blocks
def test_grouped_ffn_ragged_shapes_vs_oracle(cuda, F):
    """Shapes away from the tile sizes: F not a multiple of 256, ragged
    segments (some empty), bf16."""
    E, d = 5, 96
    counts = [0, 129, 1, 300, 70]
    start = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
    rows = int(start[-1])
    rng = np.random.default_rng(F)
    x = torch.from_numpy(rng.standard_normal((rows, d), dtype=np.float32)).to(torch.bfloat16).cuda()
    w_up = (torch.from_numpy(rng.standard_normal((E, F, d), dtype=np.float32)) / np.sqrt(d)).to(torch.bfloat16).cuda()
    w_dn = (torch.from_numpy(rng.standard_normal((E, d, F), dtype=np.float32)) / np.sqrt(F)).to(torch.bfloat16).cuda()
    mid, y = mb.grouped_ffn(x, torch.from_numpy(start).cuda(), w_up, w_dn)
    torch.cuda.synchronize()
    assert mb.device_status() == 0
    xh, wu, wd = _host16(x), _host16(w_up), _host16(w_dn)
    mh, yh = _host16(mid), _host16(y)
    for e in range(E):
        lo, hi = start[e], start[e + 1]
        if hi == lo:
            continue
        om, oy = oracle.plain_expert(xh[lo:hi], wu[e], wd[e], 1)
        gm, wm = oracle.to_f32(mh[lo:hi], 1), oracle.to_f32(om, 1)
        assert (np.abs(gm - wm) <= 1e-2 + 1e-2 * np.abs(wm)).all()   # bf16: 8 significant bits
        got, want = oracle.to_f32(yh[lo:hi], 1), oracle.to_f32(oy, 1)
        assert (np.abs(got - want) <= 1e-2 + 2e-2 * np.abs(want)).all()
