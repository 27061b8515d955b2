"""Expert-parallel host logic on CPU: world_size-2 gloo process groups.

Each rank packs its own tokens with the oracle, dispatches the packed rows
with ep.ExpertParallel (the layout from ep.layout_reference, the host
restatement of moe_b200_ep_layout), applies a per-expert transform on the
receiving side, combines the rows back and unpermutes.  The result must equal
the single-process computation, which proves every row reached the rank
owning its expert and came back to its packed position.  A second test makes
one rank fail before the exchange and checks that the other rank's collective
ends with an error instead of waiting forever."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import ep
import oracle
import routing


def join_all(ctx, seconds):
    """Waits for every spawned rank (ProcessContext.join returns after the
    first one exits); kills what is still running at the deadline and
    returns the ranks that had to be killed."""
    import time
    deadline = time.time() + seconds
    while not ctx.join(timeout=max(1.0, deadline - time.time())):
        if time.time() > deadline:
            break
    alive = [p for p in ctx.processes if p.is_alive()]
    for p in alive:
        p.kill()
    return alive


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def expert_fn(rows_f32, e):
    """A transform that depends on the global expert id."""
    return rows_f32 * (1.0 + 0.125 * e) + 0.5 * e


def _worker(rank, world, port, E, T, K, d, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        asgn, wts = routing.gen_routing(T, K, E, "zipf", seed=10 + rank)
        rng = np.random.default_rng(rank)
        embf = rng.standard_normal((T, d)).astype(np.float32)
        emb = oracle.f32_to_16(embf, 0)
        r = oracle.scatter(emb, asgn, wts, E)
        epx = ep.ExpertParallel(E, layout_fn=ep.layout_reference)
        packed = torch.from_numpy(oracle.to_f32(r["packed"], 0))
        counts = torch.from_numpy(r["expert_count"].astype(np.int32))
        recv, lay = epx.dispatch(packed, counts)
        # receiver side: apply each row's (global) expert
        ss = lay.seg_start.tolist()
        se = lay.seg_expert.tolist()
        y = torch.empty_like(recv)
        for s in range(len(se)):
            lo, hi = ss[s], ss[s + 1]
            y[lo:hi] = expert_fn(recv[lo:hi], epx.bounds[rank] + se[s])
        back = epx.combine(y, lay)
        # sender side: weighted unpermute of the returned rows
        back16 = oracle.f32_to_16(back.numpy(), 0)
        out = oracle.combine(back16, r["packed_weights"], r["slot_pos"], T, K, 0)
        # single-process reference
        want_rows = np.empty_like(back.numpy())
        starts = r["expert_start"]
        for e in range(E):
            lo, hi = starts[e], starts[e + 1]
            want_rows[lo:hi] = expert_fn(torch.from_numpy(oracle.to_f32(r["packed"][lo:hi], 0)), e).numpy()
        want = oracle.combine(oracle.f32_to_16(want_rows, 0), r["packed_weights"], r["slot_pos"], T, K, 0)
        results[rank] = (bool(np.array_equal(out, want)), lay.send, lay.recv,
                         epx.all_counts.tolist())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("E", [8, 5])  # even and uneven expert split
def test_ep_dispatch_combine_two_ranks_gloo(E):
    world, T, K, d = 2, 300, 2, 16
    port = free_port()
    with mp.Manager() as m:
        results = m.dict()
        mp.spawn(_worker, args=(world, port, E, T, K, d, results), nprocs=world, join=True)
        res = dict(results)
    assert res[0][0] and res[1][0]
    # what rank 0 sends to rank 1 is what rank 1 receives from rank 0
    assert res[0][1][1] == res[1][2][0]
    assert res[1][1][0] == res[0][2][1]
    assert res[0][3] == res[1][3]  # both gathered the same count matrix
    assert sum(res[0][1]) == T * K and sum(res[1][1]) == T * K


def _failing_worker(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    if rank == 1:
        # this rank fails on the host before the exchange and never joins it
        results[rank] = "left"
        return
    epx = ep.ExpertParallel(4, layout_fn=ep.layout_reference)
    try:
        epx.dispatch(torch.zeros((4, 8)), torch.tensor([1, 1, 1, 1], dtype=torch.int32))
        results[rank] = "completed"
    except Exception as exc:  # the collective must end with an error
        results[rank] = "error: " + type(exc).__name__


def test_ep_peer_failure_ends_in_error_not_hang():
    world = 2
    port = free_port()
    with mp.Manager() as m:
        results = m.dict()
        ctx = mp.spawn(_failing_worker, args=(world, port, results), nprocs=world, join=False)
        join_all(ctx, 120)
        res = dict(results)
    assert res.get(1) == "left"
    assert str(res.get(0, "")).startswith("error"), res


def test_layout_reference_matches_definition():
    rng = np.random.default_rng(0)
    for N, E in [(2, 8), (4, 10), (8, 60), (3, 3)]:
        counts = rng.integers(0, 50, size=(N, E)).tolist()
        b = ep.expert_ranges(E, N)
        for r in range(N):
            ss, se, send, recv = ep.layout_reference(counts, r, b)
            L = b[r + 1] - b[r]
            assert len(ss) == N * L + 1 and len(se) == N * L
            assert ss[-1] == sum(recv)
            assert sum(send) == sum(counts[r])
            for g in range(N):
                assert recv[g] == sum(counts[g][b[r]:b[r + 1]])
                for j in range(L):
                    assert ss[g * L + j + 1] - ss[g * L + j] == counts[g][b[r] + j]
                    assert se[g * L + j] == j
    assert ep.expert_ranges(60, 8) == [0, 8, 16, 24, 32, 39, 46, 53, 60]
    with pytest.raises(ValueError):
        ep.expert_ranges(3, 4)


def test_balanced_placement_is_a_permutation_that_spreads_load():
    for E, N in [(8, 2), (60, 8), (64, 4), (5, 2)]:
        lab = ep.balanced_labels(E, N)
        assert sorted(lab) == list(range(E))
        b = ep.expert_ranges(E, N)
        own = ep.placement_owner(E, N)
        for e in range(E):  # expert e lands on its owner's label range
            assert b[own[e]] <= lab[e] < b[own[e] + 1]
        # serpentine bands: the first N experts go to ranks 0..N-1, the next
        # N (where every rank still has room) to N-1..0
        assert own[:N] == list(range(N))
        if E >= 2 * N and all(b[r + 1] - b[r] >= 2 for r in range(N)):
            assert own[N:2 * N] == list(range(N - 1, -1, -1))
    # Zipf routing: the hottest rank's share drops with the balanced placement
    E, N = 60, 8
    asgn, _ = routing.gen_routing(8192, 4, E, "zipf", seed=0)
    b = ep.expert_ranges(E, N)
    def shares(a):
        c = np.bincount(a.reshape(-1), minlength=E)
        return [c[b[r]:b[r + 1]].sum() / c.sum() for r in range(N)]
    contiguous = shares(asgn)
    balanced = shares(np.asarray(ep.balanced_labels(E, N))[asgn])
    assert max(balanced) < 0.5 * max(contiguous)
