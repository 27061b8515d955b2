"""GPU tests of the fused expert-parallel path (peer-store dispatch, down-GEMM
epilogue that stores straight back to the sender, epoch flags).

With one rank the whole protocol runs against its own region, so it is
checked here on a single GPU: the output must be bit-identical to the
single-GPU layer (pack -> grouped SwiGLU -> unpermute), over several steps in
a row.  The multi-GPU test spawns one process per visible GPU (2 to 4) and is
skipped with fewer than two.  The timeout test makes a bounded wait run out
(a flag nothing sets) and checks the reported status."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch

import ep
import moe_b200 as mb
import routing

pytestmark = pytest.mark.gpu


def make_weights(E, d, I, dtype, device):
    wgu = torch.empty((E, 2 * I, d), dtype=dtype, device=device)
    wdn = torch.empty((E, d, I), dtype=dtype, device=device)
    for e in range(E):
        g = torch.Generator(device=device)
        g.manual_seed(1000 + e)
        wgu[e] = (torch.randn((2 * I, d), generator=g, device=device) * 0.02).to(dtype)
        wdn[e] = (torch.randn((d, I), generator=g, device=device) * 0.02).to(dtype)
    return wgu, wdn


def single_gpu_layer(x, a, w, E, wgu, wdn, identity):
    T, K = a.shape
    r = mb.pack(x, a, w, E)
    if identity:
        y = r.packed
    else:
        _, y = mb.grouped_swiglu(r.packed, r.expert_start, wgu, wdn)
    return mb.unpermute(y, r.packed_weights, r.slot_pos, T, K)


def run_fused_steps(epx, x, a, w, E, wgu_local, wdn_local, I, identity, steps, device, one_call=False):
    T, K = a.shape
    d = x.shape[1]
    ws = mb.Workspace(T, K, E, device=device)
    out = mb.PackResult(packed=None,
                        packed_weights=torch.empty(T * K, dtype=torch.float32, device=device),
                        perm=torch.empty(T * K, dtype=torch.int32, device=device),
                        expert_count=torch.empty(E, dtype=torch.int32, device=device),
                        expert_start=torch.empty(E + 1, dtype=torch.int32, device=device),
                        slot_pos=torch.empty(T * K, dtype=torch.int32, device=device))
    h = torch.empty((epx.recv_cap, I), dtype=x.dtype, device=device) if not identity else None
    res = []
    for _ in range(steps):
        y = torch.empty((T, d), dtype=x.dtype, device=device)
        if one_call:  # moe_b200_ep_step: the whole step in one library call
            if identity:
                epx.step(x, a, w, ws, out, y)
            else:
                epx.step(x, a, w, ws, out, y, wgu_local, wdn_local, h)
            res.append(y)
            continue
        epx.dispatch(x, a, w, ws, out)
        epx.receive()
        if identity:
            epx.return_identity()
        else:
            epx.ffn_return(wgu_local, wdn_local, h)
        epx.combine(out.packed_weights, out.slot_pos, T, y)
        res.append(y)
    torch.cuda.synchronize(device)
    return res, ws


@pytest.mark.parametrize("one_call", [False, True])
@pytest.mark.parametrize("replicated", [(), (0, 3, 5), tuple(range(16))])  # none / some / every expert
@pytest.mark.parametrize("identity", [True, False])
def test_fused_ep_single_rank_matches_single_gpu_layer(cuda, identity, replicated, one_call):
    T, K, E, d, I = 2048, 4, 16, 256, 128
    dtype = torch.bfloat16
    asgn, wts = routing.gen_routing(T, K, E, "zipf", seed=3)
    x = routing.gen_rows(T, d, "bfloat16", seed=3, device="cuda")
    a = torch.from_numpy(asgn).cuda()
    w = torch.from_numpy(wts).cuda()
    wgu, wdn = make_weights(E, d, I, dtype, "cuda")
    epx = ep.FusedExpertParallel(E, K, d, T, dtype, device="cuda", replicated=replicated)
    try:
        loc = epx.local_experts
        assert sorted(loc) == list(range(E))
        assert loc[len(loc) - len(replicated):] == sorted(replicated)
        outs, ws = run_fused_steps(epx, x, a, w, E, wgu[loc].contiguous(), wdn[loc].contiguous(), I, identity, 3,
                                   "cuda", one_call=one_call)
        assert mb.device_status() == 0
        assert ws.device_status() == 0
        want = single_gpu_layer(x, a, w, E, wgu, wdn, identity)
        for y in outs:
            assert torch.equal(y.view(torch.int16), want.view(torch.int16))
    finally:
        epx.close()


def test_custom_expert_after_receive_single_rank(cuda):
    assert _custom_expert_sees_rows(0, 1, torch.device("cuda", 0), 1024, 4, 12, 256, torch.bfloat16)
    assert mb.device_status() == 0


def test_fused_ep_wait_times_out_and_reports(cuda):
    """A flag nothing sets: the bounded wait gives up after the context's
    timeout, reports MOE_B200_DEV_WAIT_TIMEOUT, and the context stays usable."""
    T, K, E, d = 256, 2, 4, 64
    epx = ep.FusedExpertParallel(E, K, d, T, torch.float16, device="cuda", timeout_ms=100)
    try:
        assert mb.device_status() == 0
        epx.epoch = 7          # nobody raises the data flags of epoch 7
        epx.receive()
        assert mb.device_status() & mb.DEV_WAIT_TIMEOUT
        assert mb.device_status() == 0  # read-and-clear
        # a normal step afterwards works (epoch 8 > 7)
        asgn, wts = routing.gen_routing(T, K, E, "uniform", seed=1)
        x = routing.gen_rows(T, d, "float16", seed=1, device="cuda")
        a, w = torch.from_numpy(asgn).cuda(), torch.from_numpy(wts).cuda()
        outs, _ = run_fused_steps(epx, x, a, w, E, None, None, 0, True, 1, "cuda")
        assert mb.device_status() == 0
        ref = (w.sum(1, keepdim=True) * x.float())
        torch.testing.assert_close(outs[0].float(), ref, rtol=1e-3, atol=1e-3)
        # the back-flag wait inside the unpermute kernel: nobody returns rows
        # for epoch 20, so its copy warp gives up and reports
        pw = torch.full((T * K,), 0.5, dtype=torch.float32, device="cuda")
        sp = torch.arange(T * K, dtype=torch.int32, device="cuda")
        y = torch.empty((T, d), dtype=torch.float16, device="cuda")
        epx.epoch = 20
        epx.combine(pw, sp, T, y)
        assert mb.device_status() & mb.DEV_WAIT_TIMEOUT
        assert mb.device_status() == 0
        # and a one-call step still works afterwards
        outs, _ = run_fused_steps(epx, x, a, w, E, None, None, 0, True, 1, "cuda", one_call=True)
        assert mb.device_status() == 0
        torch.testing.assert_close(outs[0].float(), ref, rtol=1e-3, atol=1e-3)
    finally:
        epx.close()


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


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _custom_expert_sees_rows(rank, world, dev, T, K, E, d, dtype):
    """The stage calls with an expert kernel of the caller's own: right after
    dispatch() and receive(), a torch kernel on the same stream (no host
    synchronisation in between) sums every received row, masked on the device
    by the segment table; the sum must equal the one computed from every
    rank's inputs (regenerated here from their seeds): receive() has waited
    for every sender's rows."""
    replicated = (0, 1, 7)
    epx = ep.FusedExpertParallel(E, K, d, T, dtype, device=dev, timeout_ms=5000, replicated=replicated)
    try:
        ws = mb.Workspace(T, K, E, device=dev)
        out = mb.PackResult(packed=None,
                            packed_weights=torch.empty(T * K, dtype=torch.float32, device=dev),
                            perm=torch.empty(T * K, dtype=torch.int32, device=dev),
                            expert_count=torch.empty(E, dtype=torch.int32, device=dev),
                            expert_start=torch.empty(E + 1, dtype=torch.int32, device=dev),
                            slot_pos=torch.empty(T * K, dtype=torch.int32, device=dev))
        asgn, wts = routing.gen_routing(T, K, E, "zipf", seed=50 + rank)
        x = routing.gen_rows(T, d, "bfloat16", seed=50 + rank, device=dev)
        epx.dispatch(x, torch.from_numpy(asgn).to(dev), torch.from_numpy(wts).to(dev), ws, out)
        epx.receive()
        recv = epx.recv_rows()
        live = torch.arange(recv.shape[0], device=dev) < epx.seg_start[-1]
        got = (recv.double().sum(dim=1) * live).sum()
        mine = set(epx.local_experts[:epx.L_range])
        want = 0.0
        for s in range(world):
            a_s, _ = routing.gen_routing(T, K, E, "zipf", seed=50 + s)
            rowsum = routing.gen_rows(T, d, "bfloat16", seed=50 + s, device=dev).double().sum(dim=1).cpu().numpy()
            for t in range(T):
                for e in a_s[t]:
                    if int(e) in mine or (s == rank and int(e) in replicated):
                        want += rowsum[t]
        got = float(got.item())
        # finish the step so that every rank's buffers are released in order
        epx.return_identity()
        y = torch.empty((T, d), dtype=dtype, device=dev)
        epx.combine(out.packed_weights, out.slot_pos, T, y)
        torch.cuda.synchronize(dev)
        return abs(got - want) <= 1e-9 * max(1.0, abs(want))
    finally:
        epx.close()


def _multi_worker(rank, world, port, results):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    ok = {}
    try:
        T, K, E, d, I = 1024, 4, 12, 256, 128
        dtype = torch.bfloat16
        wgu, wdn = make_weights(E, d, I, dtype, dev)
        asgn, wts = routing.gen_routing(T, K, E, "zipf", seed=50 + rank)
        x = routing.gen_rows(T, d, "bfloat16", seed=50 + rank, device=dev)
        a, w = torch.from_numpy(asgn).to(dev), torch.from_numpy(wts).to(dev)
        # without and with replicated experts (the hottest ones: rows stay local)
        for replicated in ((), (0, 1, 7)):
            for identity in (True, False):
                epx = ep.FusedExpertParallel(E, K, d, T, dtype, device=dev, timeout_ms=5000, replicated=replicated)
                loc = epx.local_experts
                want = single_gpu_layer(x, a, w, E, wgu, wdn, identity)
                key = (identity, len(replicated))
                for one_call in (False, True):   # stage calls, then moe_b200_ep_step, on one context
                    outs, _ = run_fused_steps(epx, x, a, w, E, wgu[loc].contiguous(), wdn[loc].contiguous(), I,
                                              identity, 3, dev, one_call=one_call)
                    ok[key + (one_call,)] = all(torch.equal(y.view(torch.int16), want.view(torch.int16))
                                                for y in outs)
                ok[("status",) + key] = mb.device_status()
                epx.close()
        ok["custom_expert"] = _custom_expert_sees_rows(rank, world, dev, T, K, E, d, dtype)
        ok[("status", "custom")] = mb.device_status()
        results[rank] = ok
    finally:
        dist.barrier()
        dist.destroy_process_group()


def test_fused_ep_multi_gpu_matches_single_gpu():
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs 2 or more GPUs")
    world = min(n, 4)
    import torch.multiprocessing as mp
    with mp.Manager() as m:
        results = m.dict()
        ctx = mp.spawn(_multi_worker, args=(world, _free_port(), results), nprocs=world, join=False)
        alive = join_all(ctx, 300)
        res = dict(results)
    assert not alive, "a rank did not finish"
    for r in range(world):
        for nrep in (0, 3):
            for identity in (True, False):
                for one_call in (False, True):
                    assert res[r][(identity, nrep, one_call)], res
                assert res[r][("status", identity, nrep)] == 0, res
        assert res[r]["custom_expert"], res
        assert res[r][("status", "custom")] == 0, res
