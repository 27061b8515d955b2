"""GPU parity of the tensor-core router (moe_b200_route) against the CPU
oracle (oracle_route): gate GEMM + softmax over all experts + top-K,
replacing fused_route_kernel (apps/bench_e2e.cu:95-130).

Tolerances: the logits are a different fp32 summation order than the
reference's sequential sum, so
  - assignments must equal the oracle's wherever the oracle's K-th and
    (K+1)-th probabilities differ by more than MARGIN times the K-th
    probability (five times RTOL); a token closer to a tie than that may pick
    either expert;
  - routing weights (softmax probabilities) must match within RTOL relative,
    ATOL absolute, against the double-precision oracle (mode 1) and the
    reference's own float arithmetic (mode 0).  RTOL allows for the tensor
    cores' fp32 accumulation (hundreds of MMA steps per logit, each rounding
    its partial sum): measured worst case 2.3e-5 relative at d = 2048.
Gate weights follow the reference's fill_random_float (U(-0.05, 0.05),
include/moe/fp16_host.hpp:32-39); embeddings are N(0, 1) rounded to 16 bits.
"""
import numpy as np
import pytest
import torch

import moe_b200 as mb
import oracle

pytestmark = pytest.mark.gpu

MARGIN = 5e-4
RTOL, ATOL = 1e-4, 1e-7


def make_inputs(T, d, E, dtype, seed):
    rng = np.random.default_rng(seed)
    code = mb.dtype_code(dtype)
    emb16 = oracle.f32_to_16(rng.standard_normal((T, d)).astype(np.float32), code)
    w = rng.uniform(-0.05, 0.05, size=(d, E)).astype(np.float32)
    x = torch.from_numpy(emb16.view(np.int16)).cuda().view(dtype)
    return emb16, w, x


def check_against(a_gpu, w_gpu, a_ref, w_ref, margin):
    ok_tok = margin > MARGIN * w_ref[:, -1]
    assert ok_tok.mean() > 0.95, "too many near-ties for a meaningful test"
    assert np.array_equal(a_gpu[ok_tok], a_ref[ok_tok])
    np.testing.assert_allclose(w_gpu[ok_tok], w_ref[ok_tok], rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("T,d,E,K", [
    (1000, 512, 60, 4),    # ragged last tile, the reference's E and K
    (256, 2048, 128, 8),   # c3's E and K
    (130, 64, 8, 2),       # d below one 64-column K step
    (77, 136, 1, 1),       # a single expert, d not a multiple of 64
])
def test_route_matches_oracle(cuda, dtype, T, d, E, K):
    emb16, w, x = make_inputs(T, d, E, dtype, seed=T + d + E)
    rw = mb.RouterWeights(torch.from_numpy(w).cuda(), dtype)
    a, p = mb.route(x, rw, K)
    torch.cuda.synchronize()
    assert mb.device_status() == 0
    a, p = a.cpu().numpy(), p.cpu().numpy()
    code = mb.dtype_code(dtype)
    a1, p1, m1 = oracle.route(emb16, w, K, code, mode=1)
    check_against(a, p, a1, p1, m1)
    a0, p0, _ = oracle.route(emb16, w, K, code, mode=0)
    check_against(a, p, a0, p0, m1)


def test_route_fp16_256_experts(cuda):
    emb16, w, x = make_inputs(300, 256, 256, torch.float16, seed=7)
    rw = mb.RouterWeights(torch.from_numpy(w).cuda(), torch.float16)
    a, p = mb.route(x, rw, 8)
    a1, p1, m1 = oracle.route(emb16, w, 8, mb.F16, mode=1)
    check_against(a.cpu().numpy(), p.cpu().numpy(), a1, p1, m1)


def test_route_ties_keep_lower_index(cuda):
    """Experts 3, 5 and 6 get all-zero weight columns: their logits are
    exactly 0 whatever the accumulation order, their probabilities are equal,
    and the lower index is listed first (repeated-argmax order)."""
    T, d, E, K = 128, 128, 8, 8
    emb16, w, x = make_inputs(T, d, E, torch.bfloat16, seed=11)
    w[:, [3, 5, 6]] = 0.0
    rw = mb.RouterWeights(torch.from_numpy(w).cuda(), torch.bfloat16)
    a, p = mb.route(x, rw, K)
    a, p = a.cpu().numpy(), p.cpu().numpy()
    for t in range(T):
        row = list(a[t])
        assert sorted(row) == list(range(E))
        assert row.index(3) < row.index(5) < row.index(6)
        assert p[t, row.index(3)] == p[t, row.index(5)] == p[t, row.index(6)]


def test_route_rejects_mismatched_weights(cuda):
    emb16, w, x = make_inputs(64, 64, 16, torch.float16, seed=3)
    rw = mb.RouterWeights(torch.from_numpy(w).cuda(), torch.float16)
    mb.device_status()
    a = torch.full((64, 2), -7, dtype=torch.int32, device="cuda")
    p = torch.empty((64, 2), dtype=torch.float32, device="cuda")
    rw.E = 8                       # weights were prepared for E = 16 (same padded size)
    mb.route(x, rw, 2, out=(a, p))
    torch.cuda.synchronize()
    assert mb.device_status() & mb.DEV_BAD_WEIGHTS
    assert int(a.min()) == -7 and int(a.max()) == -7  # nothing written


def test_route_argument_errors(cuda):
    emb16, w, x = make_inputs(32, 64, 16, torch.bfloat16, seed=5)
    rw = mb.RouterWeights(torch.from_numpy(w).cuda(), torch.bfloat16)
    with pytest.raises(mb.MoEB200Error) as e:
        mb.route(x, rw, 9)
    assert e.value.status == mb.ERR_UNSUPPORTED
    with pytest.raises(mb.MoEB200Error) as e:
        mb.RouterWeights(torch.zeros((64, 200), device="cuda"), torch.bfloat16)
    assert e.value.status == mb.ERR_UNSUPPORTED
    with pytest.raises(mb.MoEB200Error) as e:
        mb.RouterWeights(torch.zeros((60, 16), device="cuda"), torch.float16)
    assert e.value.status == mb.ERR_UNSUPPORTED


def test_route_then_pack_is_bit_exact(cuda):
    """Router output feeds the packing path directly: the packed layout is
    bit-exact against cpu_scatter's restatement on the routed assignments."""
    T, d, E, K = 2048, 256, 60, 4
    emb16, w, x = make_inputs(T, d, E, torch.float16, seed=21)
    rw = mb.RouterWeights(torch.from_numpy(w).cuda(), torch.float16)
    a, p = mb.route(x, rw, K)
    r = mb.pack(x, a, p, E)
    torch.cuda.synchronize()
    ref = oracle.scatter(emb16, a.cpu().numpy(), p.cpu().numpy(), E)
    assert np.array_equal(r.packed.cpu().view(torch.int16).numpy().view(np.uint16), ref["packed"])
    assert np.array_equal(r.perm.cpu().numpy(), ref["perm"])
    assert np.array_equal(r.expert_count.cpu().numpy(), ref["expert_count"])
