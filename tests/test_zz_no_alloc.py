"""GPU test of moe_b200_pack_noalloc, the packing entry point for callers that
cannot allocate device memory (a plugin limited to its host framework's
memory pool, an FFI binding with no allocator).  It must produce exactly what
moe_b200_pack produces with a caller workspace -- packing is integer / byte
work, so the tolerance is bit equality -- on two calls in a row that share
the library's built-in scratch, and must refuse shapes whose scratch exceeds
the built-in size.  Kept in its own file, collected last."""
import ctypes

import numpy as np
import pytest
import torch

import moe_b200 as mb
import routing

pytestmark = pytest.mark.gpu

NOALLOC_SCRATCH_BYTES = 4 << 20


def noalloc_fn():
    f = mb.lib().moe_b200_pack_noalloc
    vp, ci = ctypes.c_void_p, ctypes.c_int
    f.argtypes = [vp, vp, vp, ci, ci, ci, ci, vp, vp, vp, vp, vp, vp, vp]
    f.restype = ci
    return f


def outputs(T, K, E, d, dtype):
    TK = T * K
    return dict(packed=torch.empty((TK, d), dtype=dtype, device="cuda"),
                packed_weights=torch.empty(TK, dtype=torch.float32, device="cuda"),
                perm=torch.empty(TK, dtype=torch.int32, device="cuda"),
                expert_count=torch.empty(E, dtype=torch.int32, device="cuda"),
                expert_start=torch.empty(E + 1, dtype=torch.int32, device="cuda"),
                slot_pos=torch.empty(TK, dtype=torch.int32, device="cuda"))


def call_noalloc(emb, asgn, wts, E, o):
    T, d = emb.shape
    K = asgn.shape[1]
    stream = torch.cuda.current_stream().cuda_stream
    rc = noalloc_fn()(emb.data_ptr(), asgn.data_ptr(), wts.data_ptr(), T, K, E, d,
                      o["packed"].data_ptr(), o["packed_weights"].data_ptr(), o["perm"].data_ptr(),
                      o["expert_count"].data_ptr(), o["expert_start"].data_ptr(),
                      o["slot_pos"].data_ptr(), stream)
    assert rc == mb.OK, mb.lib().moe_b200_last_error()


@pytest.mark.parametrize("T,K,E,d,dist,dtype", [
    (8192, 4, 60, 2048, "zipf", torch.float16),      # the c2 shape
    (3001, 8, 128, 72, "uniform", torch.bfloat16),   # ragged tile, E=128, K=8
])
def test_noalloc_matches_workspace_entry_point_twice(cuda, T, K, E, d, dist, dtype):
    for call in range(2):  # two calls in a row share the built-in scratch
        asgn_np, wts_np = routing.gen_routing(T, K, E, dist, seed=100 * call + T)
        emb = routing.gen_rows(T, d, "float16" if dtype == torch.float16 else "bfloat16",
                               seed=call, device="cuda")
        asgn = torch.from_numpy(asgn_np).cuda()
        wts = torch.from_numpy(wts_np).cuda()
        o = outputs(T, K, E, d, dtype)
        call_noalloc(emb, asgn, wts, E, o)
        ref = mb.pack(emb, asgn, wts, E)
        torch.cuda.synchronize()
        assert torch.equal(o["packed"].view(torch.int16), ref.packed.view(torch.int16))
        for k in ("packed_weights", "perm", "expert_count", "expert_start", "slot_pos"):
            assert torch.equal(o[k], getattr(ref, k)), k


def test_noalloc_rejects_scratch_beyond_builtin_size(cuda):
    T, K, E = (NOALLOC_SCRATCH_BYTES // 4) // 8 + 1024, 8, 64
    assert mb.pack_workspace_bytes(T, K, E) > NOALLOC_SCRATCH_BYTES
    dummy = torch.empty(16, dtype=torch.int32, device="cuda")
    p = dummy.data_ptr()
    rc = noalloc_fn()(p, p, p, T, K, E, 8, p, p, p, p, p, p, None)
    assert rc == mb.ERR_WORKSPACE
    assert b"built-in scratch" in mb.lib().moe_b200_last_error()
