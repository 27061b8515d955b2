"""Host-side Python binding of libmoe_b200 (the sm_100a MoE packing library).

Mirrors the reference's packing operator interface (feiyang-cmu/15618-final,
include/moe/types.h:18-39 and include/moe/scatter.cuh:20-65):

  MoEParams, MoEBuffers, ScatterTimings   same fields and meaning
  make_scatter(name)                      "b200" -> B200Scatter; None for
                                          unknown names (src/scatter/factory.cu:17)
  B200Scatter.name() / workspace_bytes(p) / run(d_emb, d_asgn, d_wts, bufs, p, stream)

and adds functional entry points (pack, unpermute) over the same C ABI
(include/moe_b200.h).  Tensors are torch CUDA tensors; torch provides device
memory and streams only, every kernel is in libmoe_b200.so.  Where the
reference prints and exit(1)s on a bad shape or CUDA error
(include/moe/utils.cuh:14-22), this module raises MoEB200Error.

There is no CPU fallback: if the shared library is missing, importing the
library raises.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass
from typing import NamedTuple, Optional

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "lib", "libmoe_b200.so")

OK = 0
ERR_INVALID_ARG = 1
ERR_WORKSPACE = 2
ERR_UNSUPPORTED = 3
ERR_CUDA = 4
DEV_BAD_ASSIGNMENT = 0x10
DEV_WAIT_TIMEOUT = 0x20
DEV_BAD_WEIGHTS = 0x40
F16 = 0
BF16 = 1
MAX_EXPERTS = 1024


class MoEB200Error(RuntimeError):
    """A libmoe_b200 entry point returned an error status."""

    def __init__(self, status: int, msg: str):
        super().__init__(f"{msg} (status {status})")
        self.status = status


_lib = None


def lib() -> ctypes.CDLL:
    """Load libmoe_b200.so once; raise if it was not built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise MoEB200Error(ERR_CUDA, f"libmoe_b200.so not built at {LIB_PATH}; run __graft_entry__.build()")
    L = ctypes.CDLL(LIB_PATH)
    vp, sz, i32, cint = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int32, ctypes.c_int
    L.moe_b200_version.restype = cint
    L.moe_b200_status_string.restype = ctypes.c_char_p
    L.moe_b200_status_string.argtypes = [cint]
    L.moe_b200_last_error.restype = ctypes.c_char_p
    L.moe_b200_pack_workspace_bytes.restype = sz
    L.moe_b200_pack_workspace_bytes.argtypes = [cint, cint, cint]
    L.moe_b200_workspace_init.restype = cint
    L.moe_b200_workspace_init.argtypes = [vp, sz, vp]
    L.moe_b200_pack.restype = cint
    L.moe_b200_pack.argtypes = [vp, vp, vp, cint, cint, cint, cint,
                                vp, vp, vp, vp, vp, vp, vp, sz, vp]
    L.moe_b200_workspace_status.restype = cint
    L.moe_b200_workspace_status.argtypes = [vp, sz, vp, ctypes.POINTER(cint)]
    L.moe_b200_device_status.restype = cint
    L.moe_b200_device_status.argtypes = [vp, ctypes.POINTER(cint)]
    L.moe_b200_grouped_swiglu_gather.restype = cint
    L.moe_b200_grouped_swiglu_gather.argtypes = [vp, cint, vp, vp, vp, cint, cint, cint, cint, cint, vp, vp, cint,
                                                 vp, vp, vp]
    L.moe_b200_grouped_swiglu.restype = cint
    L.moe_b200_grouped_swiglu.argtypes = [vp, vp, vp, cint, cint, cint, cint, cint, vp, vp, cint, vp, vp, vp]
    L.moe_b200_grouped_ffn.restype = cint
    L.moe_b200_grouped_ffn.argtypes = [vp, vp, vp, cint, cint, cint, cint, cint, vp, vp, cint, vp, vp, vp]
    L.moe_b200_ffn_weights_from_reference.restype = cint
    L.moe_b200_ffn_weights_from_reference.argtypes = [vp, vp, cint, cint, cint, vp, vp, vp]
    L.moe_b200_router_weights_bytes.restype = sz
    L.moe_b200_router_weights_bytes.argtypes = [cint, cint, cint]
    L.moe_b200_router_prepare.restype = cint
    L.moe_b200_router_prepare.argtypes = [vp, cint, cint, cint, vp, vp]
    L.moe_b200_route.restype = cint
    L.moe_b200_route.argtypes = [vp, cint, cint, cint, cint, cint, vp, vp, vp, vp]
    L.moe_b200_ep_layout.restype = cint
    L.moe_b200_ep_layout.argtypes = [vp, cint, cint, cint, ctypes.POINTER(ctypes.c_int32), vp, vp, vp, vp, vp]
    u64 = ctypes.c_uint64
    L.moe_b200_ep_create.restype = cint
    L.moe_b200_ep_create.argtypes = [cint, cint, cint, cint, cint, cint, ctypes.POINTER(ctypes.c_int32), cint,
                                     ctypes.POINTER(vp)]
    L.moe_b200_ep_set_replicated.restype = cint
    L.moe_b200_ep_set_replicated.argtypes = [vp, ctypes.POINTER(ctypes.c_int32), cint]
    L.moe_b200_ep_local_experts.restype = cint
    L.moe_b200_ep_local_experts.argtypes = [vp, ctypes.POINTER(ctypes.c_int32)]
    L.moe_b200_ep_destroy.restype = cint
    L.moe_b200_ep_destroy.argtypes = [vp]
    L.moe_b200_ep_ipc_handle.restype = cint
    L.moe_b200_ep_ipc_handle.argtypes = [vp, vp]
    L.moe_b200_ep_connect.restype = cint
    L.moe_b200_ep_connect.argtypes = [vp, vp]
    L.moe_b200_ep_recv_rows.restype = vp
    L.moe_b200_ep_recv_rows.argtypes = [vp]
    L.moe_b200_ep_back_rows.restype = vp
    L.moe_b200_ep_back_rows.argtypes = [vp]
    L.moe_b200_ep_recv_capacity.restype = ctypes.c_int64
    L.moe_b200_ep_recv_capacity.argtypes = [vp]
    L.moe_b200_ep_dispatch.restype = cint
    L.moe_b200_ep_dispatch.argtypes = [vp, u64, vp, vp, vp, cint, vp, vp, vp, vp, vp, vp, sz, vp]
    L.moe_b200_ep_receive.restype = cint
    L.moe_b200_ep_receive.argtypes = [vp, u64, vp, vp, vp]
    L.moe_b200_ep_return_identity.restype = cint
    L.moe_b200_ep_return_identity.argtypes = [vp, u64, vp, vp]
    L.moe_b200_ep_ffn_return.restype = cint
    L.moe_b200_ep_ffn_return.argtypes = [vp, u64, vp, vp, cint, vp, vp, cint, vp, vp]
    L.moe_b200_ep_combine.restype = cint
    L.moe_b200_ep_combine.argtypes = [vp, u64, vp, vp, cint, cint, vp, vp]
    L.moe_b200_ep_step.restype = cint
    L.moe_b200_ep_step.argtypes = [vp, vp, vp, vp, cint, cint, vp, vp, cint, vp, vp, vp, vp, vp, vp, vp, sz, vp, vp]
    L.moe_b200_ep_epoch.restype = u64
    L.moe_b200_ep_epoch.argtypes = [vp]
    L.moe_b200_unpermute.restype = cint
    L.moe_b200_unpermute.argtypes = [vp, vp, vp, cint, cint, cint, cint, vp, vp]
    _lib = L
    return L


def _check(status: int, what: str) -> None:
    if status != OK:
        L = lib()
        detail = L.moe_b200_last_error().decode() or L.moe_b200_status_string(status).decode()
        raise MoEB200Error(status, f"{what}: {detail}")


def _ptr(t) -> Optional[int]:
    if t is None:
        return None
    return t.data_ptr()


def _stream_handle(stream) -> Optional[int]:
    import torch
    if stream is None:
        stream = torch.cuda.current_stream()
    if isinstance(stream, int):
        return stream or None
    return stream.cuda_stream or None


# --------------------------------------------------------------------------
# The reference interface
# --------------------------------------------------------------------------

@dataclass
class MoEParams:
    """Problem sizes (reference include/moe/types.h:18-24)."""
    T: int
    K: int
    E: int
    d_model: int
    d_ffn: int = 0


@dataclass
class MoEBuffers:
    """Caller-owned device outputs + scratch (reference include/moe/types.h:28-39)."""
    packed: object
    packed_weights: object
    perm: object
    expert_count: object
    expert_start: object
    strategy_ws: object = None
    strategy_ws_bytes: int = 0


@dataclass
class ScatterTimings:
    """Per-stage times; 0 = not measured (reference include/moe/scatter.cuh:20-26)."""
    count_ms: float = 0.0
    prefix_ms: float = 0.0
    sort_ms: float = 0.0
    gather_ms: float = 0.0
    total_ms: float = 0.0


def allocate_buffers(p: MoEParams, device="cuda", dtype=None) -> MoEBuffers:
    """Allocate MoEBuffers the way the reference harnesses do
    (apps/bench_scatter.cu:98-113): expert_start has E+1 entries."""
    import torch
    dtype = dtype or torch.float16
    TK = p.T * p.K
    ws_bytes = pack_workspace_bytes(p.T, p.K, p.E)
    return MoEBuffers(
        packed=torch.empty((TK, p.d_model), dtype=dtype, device=device),
        packed_weights=torch.empty(TK, dtype=torch.float32, device=device),
        perm=torch.empty(TK, dtype=torch.int32, device=device),
        expert_count=torch.empty(p.E, dtype=torch.int32, device=device),
        expert_start=torch.empty(p.E + 1, dtype=torch.int32, device=device),
        strategy_ws=torch.empty(max(ws_bytes, 256), dtype=torch.uint8, device=device),
        strategy_ws_bytes=max(ws_bytes, 256),
    )


class B200Scatter:
    """The sm_100a packing strategy behind the reference's IScatter boundary."""

    def __init__(self):
        self._ws_key = None

    def name(self) -> str:
        return "b200"

    def workspace_bytes(self, p: MoEParams) -> int:
        return pack_workspace_bytes(p.T, p.K, p.E)

    def run(self, d_emb, d_asgn, d_wts, bufs: MoEBuffers, p: MoEParams, stream=None,
            slot_pos=None) -> ScatterTimings:
        s = _stream_handle(stream)
        key = (_ptr(bufs.strategy_ws), bufs.strategy_ws_bytes, p.T, p.K, p.E)
        if key != self._ws_key:
            _check(lib().moe_b200_workspace_init(_ptr(bufs.strategy_ws), bufs.strategy_ws_bytes, s),
                   "workspace_init")
            self._ws_key = key
        _check(lib().moe_b200_pack(
            _ptr(d_emb), _ptr(d_asgn), _ptr(d_wts), p.T, p.K, p.E, p.d_model,
            _ptr(bufs.packed), _ptr(bufs.packed_weights), _ptr(bufs.perm),
            _ptr(bufs.expert_count), _ptr(bufs.expert_start), _ptr(slot_pos),
            _ptr(bufs.strategy_ws), bufs.strategy_ws_bytes, s), "pack")
        return ScatterTimings()


def make_scatter(name: str):
    """Factory (reference src/scatter/factory.cu:11-18): None for unknown names."""
    if name == "b200":
        return B200Scatter()
    return None


# --------------------------------------------------------------------------
# Functional API
# --------------------------------------------------------------------------

def pack_workspace_bytes(T: int, K: int, E: int) -> int:
    return int(lib().moe_b200_pack_workspace_bytes(T, K, E))


class PackResult(NamedTuple):
    packed: object
    packed_weights: object
    perm: object
    expert_count: object
    expert_start: object
    slot_pos: object


class Workspace:
    """A zero-filled packing workspace reused across calls (one per stream)."""

    def __init__(self, T: int, K: int, E: int, device="cuda", stream=None):
        import torch
        self.nbytes = max(pack_workspace_bytes(T, K, E), 256)
        self.buf = torch.empty(self.nbytes, dtype=torch.uint8, device=device)
        self.shape = (T, K, E)
        _check(lib().moe_b200_workspace_init(self.buf.data_ptr(), self.nbytes, _stream_handle(stream)),
               "workspace_init")

    def fits(self, T, K, E) -> bool:
        return pack_workspace_bytes(T, K, E) <= self.nbytes

    def device_status(self, stream=None) -> int:
        """Synchronise and return (and clear) the device condition bits."""
        out = ctypes.c_int(0)
        _check(lib().moe_b200_workspace_status(self.buf.data_ptr(), self.nbytes,
                                               _stream_handle(stream), ctypes.byref(out)),
               "workspace_status")
        return out.value


def pack(emb, asgn, wts, E: int, workspace: Optional[Workspace] = None, out: Optional[PackResult] = None,
         stream=None, rows: bool = True) -> PackResult:
    """Stable pack of emb [T, d] (16-bit) by asgn [T, K] (int32); wts [T, K] fp32.
    rows=False: indices only (packed is None, no row copy)."""
    import torch
    T, d = emb.shape
    K = asgn.shape[1]
    TK = T * K
    dev = emb.device
    if workspace is None:
        workspace = Workspace(T, K, E, device=dev, stream=stream)
    if out is None:
        out = PackResult(
            packed=torch.empty((TK, d), dtype=emb.dtype, device=dev) if rows else None,
            packed_weights=torch.empty(TK, dtype=torch.float32, device=dev) if wts is not None else None,
            perm=torch.empty(TK, dtype=torch.int32, device=dev),
            expert_count=torch.empty(E, dtype=torch.int32, device=dev),
            expert_start=torch.empty(E + 1, dtype=torch.int32, device=dev),
            slot_pos=torch.empty(TK, dtype=torch.int32, device=dev),
        )
    _check(lib().moe_b200_pack(
        _ptr(emb), _ptr(asgn), _ptr(wts), T, K, E, d,
        _ptr(out.packed), _ptr(out.packed_weights), _ptr(out.perm),
        _ptr(out.expert_count), _ptr(out.expert_start), _ptr(out.slot_pos),
        workspace.buf.data_ptr(), workspace.nbytes, _stream_handle(stream)), "pack")
    return out


def device_status(stream=None) -> int:
    """Synchronise and return (and clear) the condition bits that workspace-less
    kernels (unpermute, grouped FFN) recorded on the current device."""
    out = ctypes.c_int(0)
    _check(lib().moe_b200_device_status(_stream_handle(stream), ctypes.byref(out)), "device_status")
    return out.value


def dtype_code(torch_dtype) -> int:
    import torch
    if torch_dtype == torch.float16:
        return F16
    if torch_dtype == torch.bfloat16:
        return BF16
    raise MoEB200Error(ERR_INVALID_ARG, f"unsupported dtype {torch_dtype}")


def unpermute(y, packed_weights, slot_pos, T: int, K: int, out=None, stream=None):
    """out[t] = round16(sum_k w[p] * y[p]), p = slot_pos[t*K + k]; fp32 accumulate."""
    import torch
    d = y.shape[1]
    if out is None:
        out = torch.empty((T, d), dtype=y.dtype, device=y.device)
    _check(lib().moe_b200_unpermute(_ptr(y), _ptr(packed_weights), _ptr(slot_pos), T, K, d,
                                    dtype_code(y.dtype), _ptr(out), _stream_handle(stream)),
           "unpermute")
    return out


def grouped_swiglu(x, seg_start, w_gate_up, w_down, seg_expert=None, h=None, y=None, stream=None,
                   row_token=None):
    """Grouped SwiGLU FFN over packed rows x [rows, d] (bf16/fp16).
    seg_start: int32 [nseg + 1] device offsets (e.g. expert_start from pack);
    w_gate_up [E, 2I, d], w_down [E, d, I].  Returns (h [rows, I], y [rows, d]).
    row_token (int32 [rows], e.g. perm from pack): x is then the token matrix
    [T, d] and packed row r is x[row_token[r]] (gathered, no packed copy)."""
    import torch
    if row_token is not None:
        T, d = x.shape
        rows = row_token.numel()
    else:
        rows, d = x.shape
    E, two_i, _ = w_gate_up.shape
    I = two_i // 2
    nseg = seg_start.numel() - 1
    if h is None:
        h = torch.empty((rows, I), dtype=x.dtype, device=x.device)
    if y is None:
        y = torch.empty((rows, d), dtype=x.dtype, device=x.device)
    if row_token is not None:
        _check(lib().moe_b200_grouped_swiglu_gather(_ptr(x), T, _ptr(row_token), _ptr(seg_start), _ptr(seg_expert),
                                                    nseg, rows, d, I, E, _ptr(w_gate_up), _ptr(w_down),
                                                    dtype_code(x.dtype), _ptr(h), _ptr(y), _stream_handle(stream)),
               "grouped_swiglu_gather")
        return h, y
    _check(lib().moe_b200_grouped_swiglu(_ptr(x), _ptr(seg_start), _ptr(seg_expert), nseg, rows, d, I, E,
                                         _ptr(w_gate_up), _ptr(w_down), dtype_code(x.dtype), _ptr(h), _ptr(y),
                                         _stream_handle(stream)), "grouped_swiglu")
    return h, y


def grouped_ffn(x, seg_start, w_up, w_down, seg_expert=None, mid=None, y=None, stream=None):
    """The reference's activation-free expert FFN, grouped, on packed rows
    x [rows, d]: mid = x . w_up[e]^T, y = mid . w_down[e]^T (fp32 accumulate,
    each rounded once).  w_up [E, F, d], w_down [E, d, F] (K-major; see
    ffn_weights_from_reference).  Returns (mid [rows, F], y [rows, d])."""
    import torch
    rows, d = x.shape
    E, F, _ = w_up.shape
    nseg = seg_start.numel() - 1
    if mid is None:
        mid = torch.empty((rows, F), dtype=x.dtype, device=x.device)
    if y is None:
        y = torch.empty((rows, d), dtype=x.dtype, device=x.device)
    _check(lib().moe_b200_grouped_ffn(_ptr(x), _ptr(seg_start), _ptr(seg_expert), nseg, rows, d, F, E, _ptr(w_up),
                                      _ptr(w_down), dtype_code(x.dtype), _ptr(mid), _ptr(y), _stream_handle(stream)),
           "grouped_ffn")
    return mid, y


def ffn_weights_from_reference(w1, w2, stream=None):
    """The reference's expert weights W1 [E, d, F] / W2 [E, F, d] (row-major
    B operands, apps/bench_e2e.cu:281-292) in the layout grouped_ffn takes:
    (w_up [E, F, d], w_down [E, d, F]), transposed on the device."""
    import torch
    E, d, F = w1.shape
    w_up = torch.empty((E, F, d), dtype=w1.dtype, device=w1.device)
    w_down = torch.empty((E, d, F), dtype=w1.dtype, device=w1.device)
    _check(lib().moe_b200_ffn_weights_from_reference(_ptr(w1.contiguous()), _ptr(w2.contiguous()), E, d, F,
                                                     _ptr(w_up), _ptr(w_down), _stream_handle(stream)),
           "ffn_weights_from_reference")
    return w_up, w_down


class RouterWeights:
    """Gate weights prepared for moe_b200_route: w_gate [d, E] fp32 on the
    device (row i = input feature i, as the reference's W_gate), split into
    16-bit pieces of the embeddings' dtype and transposed once."""

    def __init__(self, w_gate, dtype, stream=None):
        import torch
        if w_gate.dtype != torch.float32 or w_gate.dim() != 2:
            raise MoEB200Error(ERR_INVALID_ARG, "RouterWeights: w_gate must be a 2-D float32 tensor [d, E]")
        self.d, self.E = w_gate.shape
        self.dtype = dtype
        nbytes = lib().moe_b200_router_weights_bytes(self.d, self.E, dtype_code(dtype))
        if nbytes == 0:
            raise MoEB200Error(ERR_INVALID_ARG, f"RouterWeights: bad shape d={self.d} E={self.E}")
        self.buf = torch.empty(nbytes, dtype=torch.uint8, device=w_gate.device)
        _check(lib().moe_b200_router_prepare(_ptr(w_gate.contiguous()), self.d, self.E, dtype_code(dtype),
                                             _ptr(self.buf), _stream_handle(stream)), "router_prepare")


def route(x, weights, K, out=None, stream=None):
    """Router on the tensor cores: x [T, d] (bf16/fp16), weights a
    RouterWeights of the same dtype.  Returns (assignments int32 [T, K],
    routing weights fp32 [T, K]): the K most probable experts of the softmax
    over all E logits, in descending probability, ties to the lower index."""
    import torch
    T, d = x.shape
    if out is None:
        out = (torch.empty((T, K), dtype=torch.int32, device=x.device),
               torch.empty((T, K), dtype=torch.float32, device=x.device))
    _check(lib().moe_b200_route(_ptr(x), T, d, weights.E, K, dtype_code(x.dtype), _ptr(weights.buf),
                                _ptr(out[0]), _ptr(out[1]), _stream_handle(stream)), "route")
    return out


def ep_layout(all_counts, rank, expert_first, out=None, stream=None):
    """Device-side EP layout from all_counts [N, E] (int32, device).
    Returns (seg_start [N*L+1], seg_expert [N*L], send_counts [N], recv_counts [N])."""
    import torch
    N, E = all_counts.shape
    if not (0 <= rank < N) or len(expert_first) != N + 1:
        raise MoEB200Error(ERR_INVALID_ARG, f"ep_layout: rank {rank} / {len(expert_first)} bounds for {N} ranks")
    L = expert_first[rank + 1] - expert_first[rank]
    dev = all_counts.device
    if out is None:
        out = (torch.empty(N * L + 1, dtype=torch.int32, device=dev),
               torch.empty(max(N * L, 1), dtype=torch.int32, device=dev),
               torch.empty(N, dtype=torch.int32, device=dev),
               torch.empty(N, dtype=torch.int32, device=dev))
    first = (ctypes.c_int32 * (N + 1))(*expert_first)
    _check(lib().moe_b200_ep_layout(_ptr(all_counts), N, E, rank, first, _ptr(out[0]), _ptr(out[1]),
                                    _ptr(out[2]), _ptr(out[3]), _stream_handle(stream)), "ep_layout")
    return out
