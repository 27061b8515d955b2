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

from typing import List


def expert_ranges(E: int, N: int) -> List[int]:
    """First expert of every rank plus E at the end (N + 1 entries)."""
    if N < 1 or E < N:
        raise ValueError(f"need 1 <= N <= E (E={E}, N={N})")
    base, extra = divmod(E, N)
    bounds = [0]
    for r in range(N):
        bounds.append(bounds[-1] + base + (1 if r < extra else 0))
    return bounds


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
