"""ctypes binding of the CPU oracle (oracle/liboracle.so) and of the reference's
own CPU oracle when built (oracle/_ref/libref_cpu.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's cpu_baseline / --impl reference legs, never by the product path.
See moe_oracle.c for what each function restates and where it is pinned.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(_HERE, "liboracle.so")
REF_SO = os.path.join(_HERE, "_ref", "libref_cpu.so")

_P = ctypes.c_void_p
_I = ctypes.c_int
_L = ctypes.c_int64

_lib = None
_ref = None


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def build():
    subprocess.check_call(["make", "-s", "-C", _HERE, "liboracle.so"])


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(ORACLE_SO):
            build()
        L = ctypes.CDLL(ORACLE_SO)
        L.oracle_scatter.restype = _I
        L.oracle_scatter.argtypes = [_P, _P, _P, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P]
        L.oracle_verify.restype = _L
        L.oracle_verify.argtypes = [_P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I]
        L.oracle_combine.restype = None
        L.oracle_combine.argtypes = [_P, _P, _P, _I, _I, _I, _I, _P]
        L.oracle_combine_by_perm.restype = None
        L.oracle_combine_by_perm.argtypes = [_P, _P, _P, _I, _I, _I, _I, _P]
        L.oracle_swiglu_expert.restype = None
        L.oracle_swiglu_expert.argtypes = [_P, _P, _P, _I, _I, _I, _I, _P, _P]
        L.oracle_f32_to_16_array.restype = None
        L.oracle_route.argtypes = [_P, _P, _I, _I, _I, _I, _I, _I, _P, _P, _P]
        L.oracle_f32_to_16_array.argtypes = [_P, _P, _L, _I]
        L.oracle_16_to_f32_array.restype = None
        L.oracle_16_to_f32_array.argtypes = [_P, _P, _L, _I]
        L.oracle_fill_random_half.restype = None
        L.oracle_fill_random_half.argtypes = [_P, _L, ctypes.c_uint32, ctypes.c_float]
        L.oracle_fill_random_float.restype = None
        L.oracle_fill_random_float.argtypes = [_P, _L, ctypes.c_uint32, ctypes.c_float]
        L.oracle_gate_logits.restype = None
        L.oracle_gate_logits.argtypes = [_P, _P, _I, _I, _I, _I, _P]
        _lib = L
    return _lib


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def ref_lib():
    """The reference's own cpu_scatter / verify_scatter_outputs (unchanged source)."""
    global _ref
    if _ref is None:
        R = ctypes.CDLL(REF_SO)
        R.ref_cpu_scatter.restype = None
        R.ref_cpu_scatter.argtypes = [_P, _P, _P, _I, _I, _I, _I, _P, _P, _P, _P, _P]
        R.ref_verify_scatter_outputs.restype = _I
        R.ref_verify_scatter_outputs.argtypes = [_P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I]
        _ref = R
    return _ref


def _c(a, dt):
    return np.ascontiguousarray(a, dtype=dt)


def scatter(emb, asgn, wts, E):
    """Oracle pack.  emb: uint16 [T, d]; asgn int32 [T, K]; wts float32 [T, K] or None.
    Returns dict(packed, packed_weights, perm, expert_start[E+1], expert_count, slot_pos)."""
    emb = _c(emb, np.uint16)
    asgn = _c(asgn, np.int32)
    T, d = emb.shape
    K = asgn.shape[1]
    TK = T * K
    wts = None if wts is None else _c(wts, np.float32)
    out = dict(
        packed=np.empty((TK, d), np.uint16),
        packed_weights=np.empty(TK, np.float32) if wts is not None else None,
        perm=np.empty(TK, np.int32),
        expert_start=np.empty(E + 1, np.int32),
        expert_count=np.empty(E, np.int32),
        slot_pos=np.empty(TK, np.int32),
    )
    rc = lib().oracle_scatter(_p(emb), _p(asgn), _p(wts), T, K, E, d, _p(out["packed"]),
                              _p(out["packed_weights"]), _p(out["expert_start"]),
                              _p(out["expert_count"]), _p(out["perm"]), _p(out["slot_pos"]))
    if rc != 0:
        raise ValueError("assignment outside [0, E)")
    return out


def verify(emb, asgn, wts, packed, packed_w, expert_start, expert_count, perm, E) -> int:
    """Number of violated invariants (a)-(f); 0 = pass."""
    emb = _c(emb, np.uint16)
    asgn = _c(asgn, np.int32)
    T, d = emb.shape
    K = asgn.shape[1]
    return int(lib().oracle_verify(
        _p(emb), _p(asgn), _p(None if wts is None else _c(wts, np.float32)),
        _p(None if packed is None else _c(packed, np.uint16)),
        _p(None if packed_w is None else _c(packed_w, np.float32)),
        _p(_c(expert_start, np.int32)), _p(_c(expert_count, np.int32)), _p(_c(perm, np.int32)),
        T, K, E, d))


def combine(y, packed_w, slot_pos, T, K, dtype):
    """Oracle weighted unpermute: uint16 [T, d]; dtype 0 = fp16, 1 = bf16."""
    y = _c(y, np.uint16)
    d = y.shape[1]
    out = np.empty((T, d), np.uint16)
    lib().oracle_combine(_p(y), _p(_c(packed_w, np.float32)), _p(_c(slot_pos, np.int32)),
                         T, K, d, dtype, _p(out))
    return out


def combine_by_perm(y, packed_w, perm, T, dtype):
    """Reference-order (atomic-style) fp32 combine: float32 [T, d]."""
    y = _c(y, np.uint16)
    TK, d = y.shape
    out = np.empty((T, d), np.float32)
    lib().oracle_combine_by_perm(_p(y), _p(_c(packed_w, np.float32)), _p(_c(perm, np.int32)),
                                 TK, T, d, dtype, _p(out))
    return out


def swiglu_expert(x, w_gu, w_dn, dtype):
    """One SwiGLU expert on rows x (uint16 [M, D]); returns (h [M, I], y [M, D]) uint16."""
    x = _c(x, np.uint16)
    w_gu = _c(w_gu, np.uint16)
    w_dn = _c(w_dn, np.uint16)
    M, D = x.shape
    I = w_dn.shape[1]
    h = np.empty((M, I), np.uint16)
    y = np.empty((M, D), np.uint16)
    lib().oracle_swiglu_expert(_p(x), _p(w_gu), _p(w_dn), M, D, I, dtype, _p(h), _p(y))
    return h, y


def plain_expert(x, w_up, w_dn, dtype):
    """The reference's activation-free expert on rows x (uint16 [M, D]):
    w_up [F, D], w_dn [D, F]; returns (mid [M, F], y [M, D]) uint16."""
    x = _c(x, np.uint16)
    w_up = _c(w_up, np.uint16)
    w_dn = _c(w_dn, np.uint16)
    M, D = x.shape
    F = w_up.shape[0]
    mid = np.empty((M, F), np.uint16)
    y = np.empty((M, D), np.uint16)
    lib().oracle_plain_expert(_p(x), _p(w_up), _p(w_dn), M, D, F, dtype, _p(mid), _p(y))
    return mid, y


def route(emb, w_gate, K, dtype, mode=1):
    """Router oracle: emb uint16 [T, d], w_gate float32 [d, E].  mode 0 = the
    reference's float arithmetic, mode 1 = double.  Returns (assignments
    int32 [T, K], weights float32 [T, K], margin float64 [T])."""
    emb = _c(emb, np.uint16)
    w_gate = _c(w_gate, np.float32)
    T, d = emb.shape
    E = w_gate.shape[1]
    a = np.empty((T, K), np.int32)
    w = np.empty((T, K), np.float32)
    m = np.empty(T, np.float64)
    lib().oracle_route(_p(emb), _p(w_gate), T, d, E, K, dtype, mode, _p(a), _p(w), _p(m))
    return a, w, m


def fill_random_half(n, seed, half_range=0.01):
    """The reference's LCG fill (include/moe/fp16_host.hpp:22-30), fp16 bits."""
    out = np.empty(n, np.uint16)
    lib().oracle_fill_random_half(_p(out), n, seed, half_range)
    return out


def fill_random_float(n, seed, half_range=0.05):
    """The reference's LCG fill (include/moe/fp16_host.hpp:32-39)."""
    out = np.empty(n, np.float32)
    lib().oracle_fill_random_float(_p(out), n, seed, half_range)
    return out


def gate_logits(emb, w_gate, dtype=0):
    """Gate logits [T, E] in the reference's float order (sequential FMA)."""
    emb = _c(emb, np.uint16)
    w_gate = _c(w_gate, np.float32)
    T, d = emb.shape
    E = w_gate.shape[1]
    out = np.empty((T, E), np.float32)
    lib().oracle_gate_logits(_p(emb), _p(w_gate), T, d, E, dtype, _p(out))
    return out


def f32_to_16(a, dtype):
    a = _c(a, np.float32)
    out = np.empty(a.shape, np.uint16)
    lib().oracle_f32_to_16_array(_p(a), _p(out), a.size, dtype)
    return out


def to_f32(a, dtype):
    a = _c(a, np.uint16)
    out = np.empty(a.shape, np.float32)
    lib().oracle_16_to_f32_array(_p(a), _p(out), a.size, dtype)
    return out


def ref_scatter(emb, asgn, wts, E):
    """The reference's own moe::cpu_scatter (expert_start has E entries there)."""
    emb = _c(emb, np.uint16)
    asgn = _c(asgn, np.int32)
    T, d = emb.shape
    K = asgn.shape[1]
    TK = T * K
    wts = None if wts is None else _c(wts, np.float32)
    out = dict(
        packed=np.empty((TK, d), np.uint16),
        packed_weights=np.empty(TK, np.float32) if wts is not None else None,
        perm=np.empty(TK, np.int32),
        expert_start=np.empty(E, np.int32),
        expert_count=np.empty(E, np.int32),
    )
    ref_lib().ref_cpu_scatter(_p(emb), _p(asgn), _p(wts), T, K, E, d, _p(out["packed"]),
                              _p(out["packed_weights"]), _p(out["expert_start"]),
                              _p(out["expert_count"]), _p(out["perm"]))
    return out


def ref_verify(emb, asgn, wts, packed, packed_w, expert_start, expert_count, perm, E) -> bool:
    emb = _c(emb, np.uint16)
    asgn = _c(asgn, np.int32)
    T, d = emb.shape
    K = asgn.shape[1]
    return bool(ref_lib().ref_verify_scatter_outputs(
        _p(emb), _p(asgn), _p(None if wts is None else _c(wts, np.float32)),
        _p(_c(packed, np.uint16)), _p(None if packed_w is None else _c(packed_w, np.float32)),
        _p(_c(expert_start[:E], np.int32)), _p(_c(expert_count, np.int32)), _p(_c(perm, np.int32)),
        T, K, E, d))
