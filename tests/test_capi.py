"""CPU tests of the C-ABI library: it loads, exports every entry point that
include/moe_b200.h declares (plus the C++ IScatter boundary), and rejects
bad arguments on the host before touching a GPU."""
import ctypes
import os
import re
import subprocess

import pytest

import moe_b200 as mb
from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "moe_b200.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(moe_b200_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    L = mb.lib()
    names = declared_functions()
    assert len(names) >= 7
    for n in names:
        assert hasattr(L, n), n


def test_cpp_boundary_symbols_exported():
    out = subprocess.check_output(["nm", "-D", "--defined-only", mb.LIB_PATH], text=True)
    demangled = subprocess.check_output(["c++filt"], input=out, text=True)
    assert "moe::make_scatter(std::__cxx11::basic_string" in demangled
    assert "moe::make_b200_scatter()" in demangled


def test_version_and_status_strings():
    L = mb.lib()
    assert L.moe_b200_version() >= 100
    assert L.moe_b200_status_string(0) == b"ok"
    assert b"argument" in L.moe_b200_status_string(1)


def test_workspace_bytes():
    a = mb.pack_workspace_bytes(8192, 4, 60)
    assert a >= 8192 * 4 * 4 + 256
    assert a % 256 == 0
    assert mb.pack_workspace_bytes(65536, 8, 128) > a
    assert mb.pack_workspace_bytes(-1, 4, 60) == 0
    assert mb.pack_workspace_bytes(10, 0, 60) == 0


def _pack(T=16, K=2, E=4, d=8, ws=0x1000, ws_bytes=1 << 20, dev=0x2000):
    L = mb.lib()
    return L.moe_b200_pack(dev, dev, dev, T, K, E, d, dev, dev, dev, dev, dev, None, ws, ws_bytes, None)


def test_pack_rejects_bad_arguments_on_host():
    assert _pack(T=-1) == mb.ERR_INVALID_ARG
    assert _pack(K=0) == mb.ERR_INVALID_ARG
    assert _pack(E=0) == mb.ERR_INVALID_ARG
    assert _pack(d=0) == mb.ERR_INVALID_ARG
    assert _pack(K=33) == mb.ERR_UNSUPPORTED
    assert _pack(E=mb.MAX_EXPERTS + 1) == mb.ERR_UNSUPPORTED
    assert _pack(T=1 << 30, K=4) == mb.ERR_UNSUPPORTED
    assert _pack(ws_bytes=8) == mb.ERR_WORKSPACE
    assert _pack(ws=0) == mb.ERR_WORKSPACE
    assert _pack(ws=0x1010) == mb.ERR_INVALID_ARG  # not 256-byte aligned
    assert b"workspace" in mb.lib().moe_b200_last_error()


def test_unpermute_rejects_bad_arguments_on_host():
    L = mb.lib()
    p = 0x2000
    assert L.moe_b200_unpermute(p, p, p, 4, 2, 8, 7, p, None) == mb.ERR_INVALID_ARG
    assert L.moe_b200_unpermute(p, p, p, -1, 2, 8, 0, p, None) == mb.ERR_INVALID_ARG
    assert L.moe_b200_unpermute(p, p, p, 4, 40, 8, 0, p, None) == mb.ERR_UNSUPPORTED
    assert L.moe_b200_unpermute(None, p, p, 4, 2, 8, 0, p, None) == mb.ERR_INVALID_ARG
    assert L.moe_b200_unpermute(p, p, p, 0, 2, 8, 0, p, None) == mb.OK  # empty: no-op


def test_python_boundary_mirrors_reference_factory():
    assert mb.make_scatter("nope") is None
    s = mb.make_scatter("b200")
    assert s.name() == "b200"
    p = mb.MoEParams(T=2048, K=4, E=64, d_model=2048)
    assert s.workspace_bytes(p) == mb.pack_workspace_bytes(2048, 4, 64)


def test_errors_raise():
    with pytest.raises(mb.MoEB200Error) as ei:
        mb._check(mb.ERR_WORKSPACE, "x")
    assert ei.value.status == mb.ERR_WORKSPACE


def test_router_rejects_bad_arguments_on_host():
    L = mb.lib()
    p = 0x2000
    assert L.moe_b200_router_weights_bytes(2048, 60, mb.F16) == 256 + 2 * 64 * 2048 * 2
    assert L.moe_b200_router_weights_bytes(4096, 128, mb.BF16) == 256 + 3 * 128 * 4096 * 2
    assert L.moe_b200_router_weights_bytes(0, 60, mb.F16) == 0
    assert L.moe_b200_route(p, 16, 64, 16, 9, mb.F16, p, p, p, None) == mb.ERR_UNSUPPORTED   # K > 8
    assert L.moe_b200_route(p, 16, 64, 4, 5, mb.F16, p, p, p, None) == mb.ERR_UNSUPPORTED    # K > E
    assert L.moe_b200_route(p, 16, 60, 16, 2, mb.F16, p, p, p, None) == mb.ERR_UNSUPPORTED   # d % 8
    assert L.moe_b200_route(p, 16, 64, 129, 2, mb.BF16, p, p, p, None) == mb.ERR_UNSUPPORTED  # E > 128 bf16
    assert L.moe_b200_route(p, 16, 64, 16, 2, 7, p, p, p, None) == mb.ERR_INVALID_ARG        # dtype
    assert L.moe_b200_route(p, -1, 64, 16, 2, mb.F16, p, p, p, None) == mb.ERR_INVALID_ARG
    assert L.moe_b200_route(None, 16, 64, 16, 2, mb.F16, p, p, p, None) == mb.ERR_INVALID_ARG
    assert L.moe_b200_route(p + 8, 16, 64, 16, 2, mb.F16, p, p, p, None) == mb.ERR_INVALID_ARG  # alignment
    assert L.moe_b200_route(p, 0, 64, 16, 2, mb.F16, p, p, p, None) == mb.OK  # empty: no-op
    assert L.moe_b200_router_prepare(None, 64, 16, mb.F16, p, None) == mb.ERR_INVALID_ARG


def test_ep_create_rejects_bad_arguments_on_host():
    """Expert-parallel context creation validates its geometry before any
    device call (the reference asserts E % N == 0 instead,
    apps/bench_prefill.cu:361; uneven contiguous ranges are accepted here)."""
    import ctypes
    L = mb.lib()
    ctx = ctypes.c_void_p()

    def create(N=2, rank=0, E=8, K=2, d=64, max_tokens=16, first=None, timeout_ms=100):
        first = list(range(0, E + 1, E // N)) if first is None else first
        arr = (ctypes.c_int32 * len(first))(*first)
        return L.moe_b200_ep_create(N, rank, E, K, d, max_tokens, arr, timeout_ms, ctypes.byref(ctx))

    assert create(N=0, first=[0, 8]) == mb.ERR_INVALID_ARG
    assert create(rank=2) == mb.ERR_INVALID_ARG
    assert create(rank=-1) == mb.ERR_INVALID_ARG
    assert create(K=0) == mb.ERR_INVALID_ARG
    assert create(K=33) == mb.ERR_INVALID_ARG
    assert create(d=60) == mb.ERR_INVALID_ARG
    assert create(max_tokens=0) == mb.ERR_INVALID_ARG
    assert create(timeout_ms=0) == mb.ERR_INVALID_ARG
    assert create(N=4, E=2, first=[0, 1, 2, 2, 2]) == mb.ERR_INVALID_ARG        # E < N
    assert create(first=[0, 4, 7]) == mb.ERR_INVALID_ARG                        # does not end at E
    assert create(first=[1, 4, 8]) == mb.ERR_INVALID_ARG                        # does not start at 0
    assert create(first=[0, 0, 8]) == mb.ERR_INVALID_ARG                        # a rank owns nothing
    assert create(E=2048, first=[0, 1024, 2048]) == mb.ERR_UNSUPPORTED
    assert b"ep_create" in L.moe_b200_last_error()
    assert not ctx.value


def test_ep_calls_without_a_context():
    L = mb.lib()
    assert L.moe_b200_ep_set_replicated(None, None, 0) == mb.ERR_INVALID_ARG
    assert L.moe_b200_ep_local_experts(None, None) == -1
    assert L.moe_b200_ep_destroy(None) == mb.OK


def test_grouped_swiglu_rejects_bad_arguments_on_host():
    L = mb.lib()
    p = 0x2000

    def ffn(x=p, seg=p, nseg=4, rows=64, d=64, I=32, E=4, dtype=mb.BF16, h=p, y=p):
        return L.moe_b200_grouped_swiglu(x, seg, None, nseg, rows, d, I, E, p, p, dtype, h, y, None)

    assert ffn(nseg=0) == mb.ERR_INVALID_ARG
    assert ffn(rows=-1) == mb.ERR_INVALID_ARG
    assert ffn(nseg=1025) == mb.ERR_UNSUPPORTED
    assert ffn(dtype=7) == mb.ERR_INVALID_ARG
    assert ffn(d=72) == mb.ERR_UNSUPPORTED           # d % 16
    assert ffn(I=40) == mb.ERR_UNSUPPORTED           # I % 16
    assert ffn(x=None) == mb.ERR_INVALID_ARG
    assert ffn(y=None) == mb.ERR_INVALID_ARG
    assert ffn(h=p + 8) == mb.ERR_INVALID_ARG        # 16-byte alignment
    assert ffn(rows=0) == mb.OK                      # empty: no-op
    assert L.moe_b200_grouped_swiglu_gather(p, 0, p, p, None, 4, 64, 64, 32, 4, p, p, mb.BF16, p, p,
                                            None) == mb.ERR_INVALID_ARG
    assert b"grouped_swiglu" in L.moe_b200_last_error()


def _noalloc(T=16, K=2, E=4, d=8, dev=0x2000):
    L = mb.lib()
    f = L.moe_b200_pack_noalloc
    vp, ci = ctypes.c_void_p, ctypes.c_int
    f.argtypes = [vp, vp, vp, ci, ci, ci, ci, vp, vp, vp, vp, vp, vp, vp]
    f.restype = ci
    return f(dev, dev, dev, T, K, E, d, dev, dev, dev, dev, dev, None, None)


def test_noalloc_rejects_bad_arguments_on_host():
    """moe_b200_pack_noalloc's argument checks run before any CUDA call."""
    assert _noalloc(T=-1) == mb.ERR_INVALID_ARG
    assert _noalloc(K=0) == mb.ERR_INVALID_ARG
    assert _noalloc(K=33) == mb.ERR_UNSUPPORTED
    assert _noalloc(E=mb.MAX_EXPERTS + 1) == mb.ERR_UNSUPPORTED
    assert _noalloc(T=1 << 20, K=8, E=64) == mb.ERR_WORKSPACE
    assert b"built-in scratch" in mb.lib().moe_b200_last_error()
