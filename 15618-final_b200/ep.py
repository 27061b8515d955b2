"""Expert-parallel layout helpers (host side of the dispatch / combine).

Experts are split into contiguous per-rank ranges, as the reference does
(apps/bench_prefill.cu:361, apps/bench_ep.cu:16), but the split may be uneven
(E = 60 over 8 ranks gives 8,8,8,8,7,7,7,7); the reference requires E % N == 0
(bench_prefill.cu:357-360).  Because the packed rows are grouped by expert and
each rank owns a contiguous expert range, the packed buffer is already the
rank-major AllToAllv send buffer (no repack): rank g's rows are
packed[expert_start[lo_g] : expert_start[hi_g]].
"""
from __future__ import annotations

from typing import List, NamedTuple


def expert_ranges(E: int, N: int) -> List[int]:
    """First expert of every rank plus E at the end (N + 1 entries)."""
    if N < 1 or E < N:
        raise ValueError(f"need 1 <= N <= E (E={E}, N={N})")
    base, extra = divmod(E, N)
    bounds = [0]
    for r in range(N):
        bounds.append(bounds[-1] + base + (1 if r < extra else 0))
    return bounds


def placement_owner(E: int, N: int) -> List[int]:
    """Owner rank of every expert (e = popularity rank, 0 = hottest) under
    the balanced placement: experts are dealt over the ranks in serpentine
    order (0..N-1, then N-1..0, ...), skipping ranks whose label range
    (expert_ranges) is full, so every rank gets one expert of each
    popularity band and the bands alternate direction (under Zipf routing
    the busiest rank's share drops below a plain round-robin deal's)."""
    b = expert_ranges(E, N)
    cap = [b[r + 1] - b[r] for r in range(N)]
    owner = []
    band = 0
    while len(owner) < E:
        order = range(N) if band % 2 == 0 else range(N - 1, -1, -1)
        for r in order:
            if len(owner) < E and cap[r] > 0:
                owner.append(r)
                cap[r] -= 1
        band += 1
    return owner


def balanced_labels(E: int, N: int) -> List[int]:
    """Expert placement for expert parallelism: expert e (popularity rank)
    gets the next free label of rank placement_owner(E, N)[e], so rank r
    owns labels [first[r], first[r+1]).  Routing with relabelled experts is
    the same as permuting the router's output columns; packed rows stay
    grouped by owning rank."""
    b = expert_ranges(E, N)
    nxt = list(b[:-1])
    lab = []
    for r in placement_owner(E, N):
        lab.append(nxt[r])
        nxt[r] += 1
    return lab


def owner_of(E: int, N: int) -> List[int]:
    b = expert_ranges(E, N)
    own = []
    for r in range(N):
        own += [r] * (b[r + 1] - b[r])
    return own


def send_counts_from_starts(expert_start, bounds) -> List[int]:
    """Rows this rank sends to each rank g: expert_start[hi_g] - expert_start[lo_g]."""
    return [int(expert_start[bounds[g + 1]]) - int(expert_start[bounds[g]]) for g in range(len(bounds) - 1)]


def recv_layout(all_counts, bounds, rank):
    """From the gathered per-rank expert counts [N][E]: rows received from each
    sender, and the (sender, local expert) segment list of the receive buffer,
    which is sender-major then expert-major (apps/bench_prefill.cu:642-682)."""
    N = len(all_counts)
    lo, hi = bounds[rank], bounds[rank + 1]
    recv = [sum(int(all_counts[g][e]) for e in range(lo, hi)) for g in range(N)]
    segs = []
    off = 0
    for g in range(N):
        for e in range(lo, hi):
            c = int(all_counts[g][e])
            segs.append((g, e, off, c))
            off += c
    return recv, segs


def layout_reference(all_counts, rank, bounds):
    """Host restatement of moe_b200_ep_layout (used to check it and in CPU
    tests): (seg_start, seg_expert, send_counts, recv_counts) as lists."""
    N = len(all_counts)
    lo, hi = bounds[rank], bounds[rank + 1]
    send = [sum(int(all_counts[rank][e]) for e in range(bounds[g], bounds[g + 1])) for g in range(N)]
    recv, segs = recv_layout(all_counts, bounds, rank)
    seg_start = [s[2] for s in segs] + [sum(recv)]
    seg_expert = [s[1] - lo for s in segs]
    return seg_start, seg_expert, send, recv


class Layout(NamedTuple):
    seg_start: object     # device int32 [N*L + 1]
    seg_expert: object    # device int32 [N*L]
    send: List[int]       # rows sent to each rank (host)
    recv: List[int]       # rows received from each rank (host)


class ExpertParallel:
    """Dispatch / combine of packed rows across expert-parallel ranks, one
    process per GPU, over torch.distributed (NCCL on GPUs).

    dispatch: one all-gather of the E expert counts, the layout on the device
    (moe_b200_ep_layout), ONE device-to-host copy of the 2N split sizes (the
    collective library needs them on the host, as the reference's
    ncclSend/ncclRecv loop does, apps/bench_prefill.cu:768-807), then one
    AllToAllv of the rows.  The packed buffer is the send buffer.
    combine: the reverse AllToAllv, back into the sender's packed order
    (apps/bench_prefill.cu:889-906).

    `layout_fn(all_counts, rank, bounds)` may replace the device layout (the
    CPU tests inject layout_reference); by default the CUDA kernel runs."""

    def __init__(self, E: int, group=None, device=None, layout_fn=None):
        import torch
        import torch.distributed as dist
        self.dist = dist
        self.group = group
        self.N = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.E = E
        self.bounds = expert_ranges(E, self.N)
        self.L = self.bounds[self.rank + 1] - self.bounds[self.rank]
        self.device = device
        self.all_counts = torch.empty((self.N, E), dtype=torch.int32, device=device)
        self.layout_fn = layout_fn

    def exchange_counts(self, expert_count):
        self.dist.all_gather_into_tensor(self.all_counts.view(-1), expert_count[: self.E].contiguous(),
                                         group=self.group)
        return self.all_counts

    def layout(self, expert_count) -> Layout:
        import torch
        counts = self.exchange_counts(expert_count)
        if self.layout_fn is None:
            import moe_b200 as mb
            seg_start, seg_expert, send, recv = mb.ep_layout(counts, self.rank, self.bounds)
            host = torch.stack([send, recv]).cpu()
            return Layout(seg_start, seg_expert, host[0].tolist(), host[1].tolist())
        ss, se, send, recv = self.layout_fn(counts.cpu().tolist(), self.rank, self.bounds)
        return Layout(torch.tensor(ss, dtype=torch.int32, device=self.device),
                      torch.tensor(se, dtype=torch.int32, device=self.device), send, recv)

    def dispatch(self, packed, expert_count, recv_buf=None):
        """Returns (rows received [sum(recv), d] in sender-major / expert-major
        order, layout)."""
        import torch
        lay = self.layout(expert_count)
        nrecv = sum(lay.recv)
        if recv_buf is None or recv_buf.shape[0] < nrecv:
            recv_buf = torch.empty((nrecv, packed.shape[1]), dtype=packed.dtype, device=packed.device)
        out = recv_buf[:nrecv]
        self.dist.all_to_all_single(out, packed[: sum(lay.send)], lay.recv, lay.send, group=self.group)
        return out, lay

    def combine(self, y, lay: Layout, back=None):
        """Sends expert outputs y (receive order) back; returns rows aligned with
        this rank's packed buffer."""
        import torch
        nsend = sum(lay.send)
        if back is None or back.shape[0] < nsend:
            back = torch.empty((nsend, y.shape[1]), dtype=y.dtype, device=y.device)
        out = back[:nsend]
        self.dist.all_to_all_single(out, y[: sum(lay.recv)], lay.send, lay.recv, group=self.group)
        return out


class _DeviceArray:
    """Exposes a raw device allocation to torch (zero copy)."""

    def __init__(self, ptr, shape, typestr):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (int(ptr), False),
                                         "version": 3, "strides": None}


class FusedExpertParallel:
    """Expert parallelism without a collective library on the data path: the
    packing kernel stores each token row straight into the receive buffer of
    the rank owning its expert (peer memory over NVLink, mapped with CUDA IPC),
    the expert's down-GEMM stores its rows straight back into the sender's
    buffer, and epoch flags in peer memory order the steps.  torch.distributed
    is used once, to exchange the 64-byte IPC handles.  See include/moe_b200.h
    (moe_b200_ep_*) for the protocol; replaces the reference's host-synchronised
    NCCL exchange (apps/bench_prefill.cu:768-807, 889-906).

    Every rank must run the same sequence of steps (epochs advance together).

    `replicated`: global expert ids every rank holds a copy of (the same list
    on every rank); their rows never leave their rank.  `local_experts` lists
    the global ids of this rank's expert weights in the order ffn_return
    expects: the non-replicated experts of its range, then the replicated
    ones."""

    def __init__(self, E: int, K: int, d: int, max_tokens: int, dtype, group=None, device=None,
                 timeout_ms: int = 2000, replicated=()):
        import ctypes
        import torch
        import torch.distributed as dist
        import moe_b200 as mb
        self.mb = mb
        self.L_ = mb.lib()
        self.dist = dist
        self.group = group
        if dist.is_available() and dist.is_initialized():
            self.N, self.rank = dist.get_world_size(group), dist.get_rank(group)
        else:
            self.N, self.rank = 1, 0
        self.E, self.K, self.d, self.dtype = E, K, d, dtype
        self.bounds = expert_ranges(E, self.N)
        self.L = self.bounds[self.rank + 1] - self.bounds[self.rank]
        self.device = device
        first = (ctypes.c_int32 * (self.N + 1))(*self.bounds)
        self.ctx = ctypes.c_void_p()
        mb._check(self.L_.moe_b200_ep_create(self.N, self.rank, E, K, d, max_tokens, first, timeout_ms,
                                             ctypes.byref(self.ctx)), "ep_create")
        rep_ids = sorted(set(int(e) for e in replicated))
        arr = (ctypes.c_int32 * max(1, len(rep_ids)))(*rep_ids)
        mb._check(self.L_.moe_b200_ep_set_replicated(self.ctx, arr, len(rep_ids)), "ep_set_replicated")
        self.replicated = rep_ids
        n_local = self.L_.moe_b200_ep_local_experts(self.ctx, None)
        loc = (ctypes.c_int32 * n_local)()
        self.L_.moe_b200_ep_local_experts(self.ctx, loc)
        self.local_experts = list(loc)
        self.L_range = n_local - len(rep_ids)   # non-replicated experts of this rank's range
        h = (ctypes.c_uint8 * 64)()
        mb._check(self.L_.moe_b200_ep_ipc_handle(self.ctx, h), "ep_ipc_handle")
        mine = torch.tensor(list(h), dtype=torch.uint8, device=device)
        if self.N > 1:
            allh = torch.empty(self.N * 64, dtype=torch.uint8, device=device)
            dist.all_gather_into_tensor(allh, mine, group=group)
        else:
            allh = mine
        buf = (ctypes.c_uint8 * (self.N * 64))(*allh.cpu().tolist())
        mb._check(self.L_.moe_b200_ep_connect(self.ctx, buf), "ep_connect")
        self.epoch = 0
        nseg = n_local   # one receive segment per local expert (expert-major receive buffer)
        mk = lambda n: torch.empty(n, dtype=torch.int32, device=device)
        self.seg_start, self.seg_expert = mk(nseg + 1), mk(nseg)
        self.recv_cap = int(self.L_.moe_b200_ep_recv_capacity(self.ctx))

    def _s(self, stream):
        return self.mb._stream_handle(stream)

    def recv_rows(self):
        import torch
        p = self.L_.moe_b200_ep_recv_rows(self.ctx)
        return torch.as_tensor(_DeviceArray(p, (self.recv_cap, self.d), "<i2"), device=self.device).view(self.dtype)

    def step(self, emb, asgn, wts, workspace, out, y, w_gate_up=None, w_down=None, h=None, stream=None):
        """One whole step in ONE library call (moe_b200_ep_step): pack +
        dispatch, receive, the expert (identity when no weights are given,
        else the grouped SwiGLU with w_gate_up / w_down / h as ffn_return),
        return and combine into y [T, d].  `out` is a moe_b200.PackResult
        (packed unused)."""
        T = emb.shape[0]
        p = self.mb._ptr
        I = 0 if w_down is None else w_down.shape[2]
        self.mb._check(self.L_.moe_b200_ep_step(
            self.ctx, p(emb), p(asgn), p(wts), T, I, p(w_gate_up), p(w_down), self.mb.dtype_code(self.dtype), p(h),
            p(out.packed_weights), p(out.perm), p(out.expert_count), p(out.expert_start), p(out.slot_pos),
            workspace.buf.data_ptr(), workspace.nbytes, p(y), self._s(stream)), "ep_step")
        self.epoch = int(self.L_.moe_b200_ep_epoch(self.ctx))

    def dispatch(self, emb, asgn, wts, workspace, out, stream=None):
        """Starts a step: pack + peer-store dispatch.  `out` is a moe_b200.PackResult
        (its packed buffer is not written: rows go straight to their owners)."""
        self.epoch = max(self.epoch, int(self.L_.moe_b200_ep_epoch(self.ctx))) + 1
        T = emb.shape[0]
        p = self.mb._ptr
        self.mb._check(self.L_.moe_b200_ep_dispatch(
            self.ctx, self.epoch, p(emb), p(asgn), p(wts), T, p(out.packed_weights), p(out.perm),
            p(out.expert_count), p(out.expert_start), p(out.slot_pos), workspace.buf.data_ptr(), workspace.nbytes,
            self._s(stream)), "ep_dispatch")

    def receive(self, stream=None):
        p = self.mb._ptr
        self.mb._check(self.L_.moe_b200_ep_receive(self.ctx, self.epoch, p(self.seg_start), p(self.seg_expert),
                                                   self._s(stream)), "ep_receive")

    def return_identity(self, stream=None):
        p = self.mb._ptr
        self.mb._check(self.L_.moe_b200_ep_return_identity(self.ctx, self.epoch, p(self.seg_start),
                                                           self._s(stream)), "ep_return_identity")

    def ffn_return(self, w_gate_up, w_down, h, stream=None):
        """Grouped SwiGLU on the received rows: w_gate_up [n, 2I, d] /
        w_down [n, d, I] for the n = len(local_experts) local experts in
        local_experts order; h: [recv_capacity, I] scratch."""
        p = self.mb._ptr
        I = w_down.shape[2]
        self.mb._check(self.L_.moe_b200_ep_ffn_return(
            self.ctx, self.epoch, p(self.seg_start), p(self.seg_expert), I, p(w_gate_up), p(w_down),
            self.mb.dtype_code(self.dtype), p(h), self._s(stream)), "ep_ffn_return")

    def combine(self, packed_weights, slot_pos, T, out, stream=None):
        p = self.mb._ptr
        self.mb._check(self.L_.moe_b200_ep_combine(self.ctx, self.epoch, p(packed_weights), p(slot_pos), T,
                                                   self.mb.dtype_code(self.dtype), p(out), self._s(stream)),
                       "ep_combine")

    def close(self):
        if self.ctx:
            import torch
            torch.cuda.synchronize()
            if self.N > 1:
                self.dist.barrier(group=self.group)
            self.L_.moe_b200_ep_destroy(self.ctx)
            self.ctx = None
