"""GPU numerics of the tcgen05 grouped SwiGLU FFN (through the C ABI).

References: a plain PyTorch fp32 computation of the same op, and the C oracle
(oracle_swiglu_expert, double accumulation) on small cases.  Tolerances are
for 16-bit outputs of an fp32-accumulated GEMM: each GEMM is checked against
an fp32 reference fed the kernel's own inputs (so bf16 rounding of h is not
double counted), with |err| <= RTOL * |ref| + ATOL * max|ref|."""
import numpy as np
import pytest
import torch

import moe_b200 as mb
import oracle
import routing

pytestmark = pytest.mark.gpu

RTOL = {torch.bfloat16: 2e-2, torch.float16: 4e-3}
ATOL = {torch.bfloat16: 1e-2, torch.float16: 2e-3}


def close(got, ref, dtype):
    got = got.float()
    ref = ref.float()
    scale = ref.abs().max().item() + 1e-12
    err = (got - ref).abs()
    bound = RTOL[dtype] * ref.abs() + ATOL[dtype] * scale
    bad = (err > bound).sum().item()
    assert bad == 0, f"{bad} of {ref.numel()} elements out of tolerance; max err {err.max().item():.3g}, scale {scale:.3g}"


def torch_ffn(x, seg_start, seg_expert, wgu, wdn, h_gpu):
    """fp32 reference of both GEMMs; GEMM 2 is fed the kernel's own h."""
    I = wdn.shape[2]
    h_ref = torch.zeros((x.shape[0], I), dtype=torch.float32, device=x.device)
    y_ref = torch.zeros((x.shape[0], wdn.shape[1]), dtype=torch.float32, device=x.device)
    ss = seg_start.tolist()
    for s in range(len(ss) - 1):
        lo, hi = ss[s], ss[s + 1]
        if hi <= lo:
            continue
        e = seg_expert[s] if seg_expert is not None else s
        xs = x[lo:hi].float()
        g = xs @ wgu[e, :I].float().T
        u = xs @ wgu[e, I:].float().T
        h_ref[lo:hi] = torch.nn.functional.silu(g) * u
        y_ref[lo:hi] = h_gpu[lo:hi].float() @ wdn[e].float().T
    return h_ref, y_ref


def make_problem(counts, d, I, dtype, seed=0, E=None):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    E = E or len(counts)
    rows = int(sum(counts))
    x = torch.randn((rows, d), generator=g, device="cuda").to(dtype)
    wgu = (torch.randn((E, 2 * I, d), generator=g, device="cuda") * 0.02).to(dtype)
    wdn = (torch.randn((E, d, I), generator=g, device="cuda") * 0.02).to(dtype)
    seg = torch.tensor(np.concatenate([[0], np.cumsum(counts)]).astype(np.int32), device="cuda")
    return x, wgu, wdn, seg


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("counts,d,I", [
    ([200, 0, 77], 256, 128),          # empty expert, partial row blocks
    ([1, 129, 255, 256], 128, 192),    # partial N block in GEMM 1 (I = 1.5 x 128)
    ([513], 512, 256),
    ([40, 300, 0, 0, 17, 1000], 320, 96),  # d not a multiple of 256: partial N block in GEMM 2
])
def test_grouped_swiglu_vs_torch_fp32(cuda, counts, d, I, dtype):
    x, wgu, wdn, seg = make_problem(counts, d, I, dtype)
    h, y = mb.grouped_swiglu(x, seg, wgu, wdn)
    assert mb.device_status() == 0
    h_ref, y_ref = torch_ffn(x, seg, None, wgu, wdn, h)
    close(h, h_ref, dtype)
    close(y, y_ref, dtype)


def test_grouped_swiglu_vs_oracle_small(cuda):
    counts, d, I, dtype = [70, 130], 128, 64, torch.bfloat16
    x, wgu, wdn, seg = make_problem(counts, d, I, dtype, seed=3)
    h, y = mb.grouped_swiglu(x, seg, wgu, wdn)
    torch.cuda.synchronize()
    bits = lambda t: t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
    ss = seg.tolist()
    for e in range(len(counts)):
        lo, hi = ss[e], ss[e + 1]
        ho, yo = oracle.swiglu_expert(bits(x[lo:hi]), bits(wgu[e]), bits(wdn[e]), 1)
        close(h[lo:hi], torch.from_numpy(oracle.to_f32(ho, 1)).cuda(), dtype)
        # end to end through both roundings: twice the single-GEMM tolerance
        ref = torch.from_numpy(oracle.to_f32(yo, 1)).cuda()
        got = y[lo:hi].float()
        scale = ref.abs().max().item()
        assert ((got - ref).abs() <= 2 * (RTOL[dtype] * ref.abs() + ATOL[dtype] * scale)).all()


def test_grouped_swiglu_segments_with_expert_map(cuda):
    """EP receive layout: segments are (sender, local expert) runs, experts repeat."""
    counts = [50, 0, 130, 20, 64, 1]
    seg_expert = [1, 0, 1, 2, 0, 2]
    d, I, dtype = 256, 128, torch.bfloat16
    x, wgu, wdn, seg = make_problem(counts, d, I, dtype, seed=5, E=3)
    se = torch.tensor(seg_expert, dtype=torch.int32, device="cuda")
    h, y = mb.grouped_swiglu(x, seg, wgu, wdn, seg_expert=se)
    assert mb.device_status() == 0
    h_ref, y_ref = torch_ffn(x, seg, seg_expert, wgu, wdn, h)
    close(h, h_ref, dtype)
    close(y, y_ref, dtype)


def test_pack_ffn_unpermute_layer_c5_shape(cuda):
    """The full single-GPU layer at the c5 shape: pack -> grouped SwiGLU -> unpermute,
    checked on a sample of tokens against an fp32 torch layer."""
    c = routing.CONFIGS["c5"]
    T, K, E, d, I = c["T"], c["K"], c["E"], c["d"], c["I"]
    dtype = torch.bfloat16
    asgn, wts = routing.gen_routing(T, K, E, c["dist"], c["seed"])
    x = routing.gen_rows(T, d, "bfloat16", c["seed"], device="cuda")
    g = torch.Generator(device="cuda")
    g.manual_seed(11)
    wgu = (torch.randn((E, 2 * I, d), generator=g, device="cuda") * 0.02).to(dtype)
    wdn = (torch.randn((E, d, I), generator=g, device="cuda") * 0.02).to(dtype)
    a = torch.from_numpy(asgn).cuda()
    w = torch.from_numpy(wts).cuda()
    r = mb.pack(x, a, w, E)
    h, y = mb.grouped_swiglu(r.packed, r.expert_start, wgu, wdn)
    out = mb.unpermute(y, r.packed_weights, r.slot_pos, T, K)
    assert mb.device_status() == 0
    # every GEMM row against fp32 on a sample of experts (incl. the hottest)
    h_ref, y_ref = torch_ffn(r.packed, r.expert_start, None, wgu, wdn, h)
    for e in [0, 1, 7, 31, E - 1]:
        lo, hi = r.expert_start[e].item(), r.expert_start[e + 1].item()
        close(h[lo:hi], h_ref[lo:hi], dtype)
        close(y[lo:hi], y_ref[lo:hi], dtype)
    # combined output of 256 sampled tokens vs an fp32 torch layer using the kernel's y
    idx = torch.randperm(T, generator=torch.Generator().manual_seed(0))[:256].cuda()
    sp = r.slot_pos.view(T, K)[idx].long()
    ref = (w[idx].unsqueeze(-1) * y[sp].float()).sum(1)
    close(out[idx], ref, dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("T,K,E,d,I,dist", [
    (2048, 4, 16, 256, 128, "zipf"),
    (1001, 3, 7, 128, 256, "uniform"),     # ragged segments and tile tails
    (300, 8, 40, 64, 64, "uniform"),       # many small segments, d = one K step
])
def test_grouped_swiglu_gather_matches_packed(cuda, dtype, T, K, E, d, I, dist):
    """Gathered form (A rows fetched from the token matrix with tile::gather4
    by perm, pack run with packed = NULL) == the packed form, bit for bit."""
    asgn, wts = routing.gen_routing(T, K, E, dist, seed=T)
    g = torch.Generator(device="cuda")
    g.manual_seed(T)
    x = torch.randn((T, d), generator=g, device="cuda").to(dtype)
    wgu = (torch.randn((E, 2 * I, d), generator=g, device="cuda") * 0.02).to(dtype)
    wdn = (torch.randn((E, d, I), generator=g, device="cuda") * 0.02).to(dtype)
    a = torch.from_numpy(asgn).cuda()
    w = torch.from_numpy(wts).cuda()
    full = mb.pack(x, a, w, E)
    idx = mb.pack(x, a, w, E, rows=False)
    assert idx.packed is None
    for f in ("perm", "packed_weights", "expert_count", "expert_start", "slot_pos"):
        assert torch.equal(getattr(full, f), getattr(idx, f)), f
    h1, y1 = mb.grouped_swiglu(full.packed, full.expert_start, wgu, wdn)
    h2, y2 = mb.grouped_swiglu(x, idx.expert_start, wgu, wdn, row_token=idx.perm)
    torch.cuda.synchronize()
    assert mb.device_status() == 0
    assert torch.equal(h1.view(torch.int16), h2.view(torch.int16))
    assert torch.equal(y1.view(torch.int16), y2.view(torch.int16))
