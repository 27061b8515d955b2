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


def test_noalloc_shrinking_then_growing_shapes(cuda):
    """Consecutive calls with shrinking then growing (T, K, E): a large plan
    leaves look-back words past a smaller plan's clear, so every call must
    still match moe_b200_pack with a fresh workspace bit for bit."""
    for T, K, E, d in ((3001, 8, 128, 72), (257, 2, 8, 64), (8192, 4, 60, 2048), (40, 1, 3, 16),
                       (4096, 8, 128, 128)):
        asgn_np, wts_np = routing.gen_routing(T, K, E, "zipf", seed=T + E)
        emb = routing.gen_rows(T, d, "float16", seed=K, device="cuda")
        asgn = torch.from_numpy(asgn_np).cuda()
        wts = torch.from_numpy(wts_np).cuda()
        o = outputs(T, K, E, d, torch.float16)
        call_noalloc(emb, asgn, wts, E, o)
        ref = mb.pack(emb, asgn, wts, E, workspace=mb.Workspace(T, K, E))
        torch.cuda.synchronize()
        assert torch.equal(o["packed"].view(torch.int16), ref.packed.view(torch.int16)), (T, K, E)
        for k in ("packed_weights", "perm", "expert_count", "expert_start", "slot_pos"):
            assert torch.equal(o[k], getattr(ref, k)), (k, T, K, E)


FIRST_CALL_SCRIPT = r'''
import os, sys
sys.path[:0] = sys.argv[1].split(os.pathsep)
import torch, routing, moe_b200 as mb
import test_zz_no_alloc as t
T, K, E, d = 2048, 4, 60, 256
s = torch.cuda.Stream()          # a non-blocking stream, the process's first library call
asgn_np, wts_np = routing.gen_routing(T, K, E, "zipf", seed=7)
with torch.cuda.stream(s):
    emb = routing.gen_rows(T, d, "float16", seed=7, device="cuda")
    asgn = torch.from_numpy(asgn_np).cuda()
    wts = torch.from_numpy(wts_np).cuda()
    o = t.outputs(T, K, E, d, torch.float16)
    t.call_noalloc(emb, asgn, wts, E, o)
    ref = mb.pack(emb, asgn, wts, E)
s.synchronize()
ok = torch.equal(o["packed"].view(torch.int16), ref.packed.view(torch.int16)) and all(
    torch.equal(o[k], getattr(ref, k)) for k in ("packed_weights", "perm", "expert_count", "expert_start",
                                                  "slot_pos"))
print("FIRST_CALL_OK" if ok else "FIRST_CALL_MISMATCH")
'''


def test_noalloc_first_call_on_nonblocking_stream(cuda):
    """The process's very first call (the set-up) made on a non-blocking
    stream, in a fresh process, matches the workspace entry point."""
    import os
    import subprocess
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    pkg = os.path.join(os.path.dirname(here), "15618-final_b200")
    r = subprocess.run([sys.executable, "-c", FIRST_CALL_SCRIPT, pkg + os.pathsep + here], capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    assert "FIRST_CALL_OK" in r.stdout, r.stdout[-2000:]


def test_noalloc_empty_batch(cuda):
    o = outputs(1, 4, 60, 64, torch.float16)
    emb = torch.empty((0, 64), dtype=torch.float16, device="cuda")
    asgn = torch.empty((0, 4), dtype=torch.int32, device="cuda")
    wts = torch.empty((0, 4), dtype=torch.float32, device="cuda")
    call_noalloc(emb, asgn, wts, 60, o)
    torch.cuda.synchronize()


def test_noalloc_rejects_scratch_beyond_builtin_size(cuda):
    T, K, E = (NOALLOC_SCRATCH_BYTES // 4) // 8 + 1024, 8, 64
    assert mb.pack_workspace_bytes(T, K, E) > NOALLOC_SCRATCH_BYTES
    dummy = torch.empty(16, dtype=torch.int32, device="cuda")
    p = dummy.data_ptr()
    rc = noalloc_fn()(p, p, p, T, K, E, 8, p, p, p, p, p, p, None)
    assert rc == mb.ERR_WORKSPACE
    assert b"built-in scratch" in mb.lib().moe_b200_last_error()
