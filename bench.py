"""Benchmark of the MoE token packing + weighted unpermute path.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--config c2]

One step = one pass of the hot path over one batch:
  N = 1   pack (route_scan + pack_rows) -> identity expert -> unpermute, on the
          single-B200 workload (config c2: T=8192, d=2048 fp16, E=60, K=4,
          Zipf s=1.2 routing).
  N > 1   (torchrun, one rank per GPU, NCCL) each rank packs its own T=8192
          tokens, AllToAllv-dispatches the packed rows to the expert-owning
          ranks, applies the identity expert, AllToAllv-combines them back and
          unpermutes: weak scaling, value = all ranks' tokens / max-rank time.

Prints ONE JSON line on rank 0.  `value` is device-timed (CUDA events on the
launching stream, inputs resident in HBM, L2 flushed by a 256 MiB write + a
256 MiB read before every step); `e2e` is the same metric through the C ABI with pinned host
buffers and the host<->device copies inside the timed region.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [os.path.join(ROOT, "15618-final_b200")]

import numpy as np  # noqa: E402

import routing  # noqa: E402

METRIC = "scatter+unpermute tokens/s"
UNIT = "tokens/s"
FALLBACK_HBM_GBS = 6650.0


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--config", default="c2", choices=["c1", "c2", "c3", "c4"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    return ap.parse_args()


def workload(cfg_name, rank=0):
    c = dict(routing.CONFIGS[cfg_name])
    c["seed"] = c["seed"] + rank
    return c


def config_json(c, n, l2_note):
    return {
        "workload": f"{c['name']}: T={c['T']} per GPU, d={c['d']} {c['dtype']}, E={c['E']}, "
                    f"K={c['K']}, {c['dist']} routing" + (" s=1.2" if c["dist"] == "zipf" else ""),
        "T_per_gpu": c["T"], "d": c["d"], "E": c["E"], "K": c["K"], "routing": c["dist"],
        "expert": "identity",
        "pipeline": "pack -> unpermute" if n == 1 else "pack -> AllToAllv -> identity -> AllToAllv -> unpermute",
        "parallelism": f"ep{n}" if n > 1 else "single-gpu",
        "l2": l2_note,
    }


def algorithmic_bytes(c):
    T, d, K, E = c["T"], c["d"], c["K"], c["E"]
    s = 2
    TK = T * K
    b_pack = T * d * s + TK * d * s + TK * 8 + TK * 8 + 8 * E
    b_unperm = TK * d * s + TK * 8 + T * d * s
    return b_pack, b_unperm


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def committed_traffic(kernel, workload_name):
    path = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(path) as f:
            return json.load(f).get(f"{kernel}@{workload_name}")
    except Exception:
        return None


# --------------------------------------------------------------- clocks ----

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.lines:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------- L2 flush ----

L2_NOTE = ("flushed before every step: 256 MiB write, then a 256 MiB read, so L2 holds none of "
           "the step's data and no dirty lines")


class L2Flush:
    """Writes a 256 MiB buffer (2x the 126 MB L2), then reads another one so the
    written lines are evicted (and written back) before the timed step starts."""

    def __init__(self, dev):
        import torch
        self.w = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
        self.r = torch.ones(64 << 20, dtype=torch.float32, device=dev)
        self.sink = torch.empty((), dtype=torch.float32, device=dev)

    def __call__(self, i):
        import torch
        self.w.fill_(i & 0xFF)
        torch.sum(self.r, dim=0, out=self.sink)


# ----------------------------------------------------------- CPU legs -----

def cpu_inputs(c, T_sample):
    import torch
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    asgn, wts = routing.gen_routing(c["T"], c["K"], c["E"], c["dist"], c["seed"])
    rows = routing.gen_rows(T_sample, c["d"], c["dtype"], c["seed"])
    emb = rows.view(torch.int16).numpy().view(np.uint16)
    return emb, np.ascontiguousarray(asgn[:T_sample]), np.ascontiguousarray(wts[:T_sample])


class CpuWorker:
    """One host thread's buffers for the CPU path: the reference's own
    moe::cpu_scatter (oracle/_ref, unchanged source) when built here, else the
    oracle restatement; then the oracle combine (the reference has no CPU
    combine).  ctypes drops the GIL, so threads run in parallel."""

    def __init__(self, emb, asgn, wts, E, dtype_code):
        import oracle
        self.o = oracle
        self.emb, self.asgn, self.wts, self.E, self.dt = emb, asgn, wts, E, dtype_code
        T, d = emb.shape
        K = asgn.shape[1]
        self.T, self.K, self.d = T, K, d
        self.packed = np.zeros((T * K, d), np.uint16)
        self.pw = np.zeros(T * K, np.float32)
        self.perm = np.zeros(T * K, np.int32)
        self.start = np.zeros(E + 1, np.int32)
        self.count = np.zeros(E, np.int32)
        self.slot_pos = np.zeros(T * K, np.int32)
        self.out = np.zeros((T, d), np.uint16)
        r = oracle.scatter(emb, asgn, wts, E)  # slot_pos (inverse of perm) for the combine
        self.slot_pos[:] = r["slot_pos"]
        self.use_ref = oracle.ref_available()
        self.kind = "reference" if self.use_ref else "port"

    def step(self):
        p = self.o._p
        if self.use_ref:
            self.o.ref_lib().ref_cpu_scatter(p(self.emb), p(self.asgn), p(self.wts), self.T, self.K, self.E,
                                             self.d, p(self.packed), p(self.pw), p(self.start), p(self.count),
                                             p(self.perm))
        else:
            self.o.lib().oracle_scatter(p(self.emb), p(self.asgn), p(self.wts), self.T, self.K, self.E, self.d,
                                        p(self.packed), p(self.pw), p(self.start), p(self.count), p(self.perm),
                                        p(self.slot_pos))
        self.o.lib().oracle_combine(p(self.packed), p(self.pw), p(self.slot_pos), self.T, self.K, self.d,
                                    self.dt, p(self.out))


def run_cpu(c, threads, T_sample, steps, warmup, min_seconds=0.0):
    """Returns (tokens/s over all threads, seconds per step, kind).  With
    min_seconds, the step count grows until the timed work lasts that long."""
    emb, asgn, wts = cpu_inputs(c, T_sample)
    dt = 0 if c["dtype"] == "float16" else 1
    workers = [CpuWorker(emb, asgn, wts, c["E"], dt) for _ in range(threads)]
    for _ in range(max(warmup, 1)):
        t0 = time.perf_counter()
        for w in workers:
            w.step()
        one = (time.perf_counter() - t0) / threads
    if min_seconds > 0:
        steps = max(steps, min(400, int(min_seconds / max(one, 1e-6)) + 1))
    times = []
    for _ in range(steps):
        ths = [threading.Thread(target=w.step) for w in workers]
        t0 = time.perf_counter()
        for th in ths:
            th.start()
        for th in ths:
            th.join()
        times.append(time.perf_counter() - t0)
    total = sum(times)
    return threads * T_sample * steps / total, total / steps, workers[0].kind


def host_cores():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    c = workload(args.config)
    c["name"] = args.config
    cores = host_cores()
    T_sample = min(c["T"], 2048)
    warm = max(args.warmup, 3)
    steps = max(1, min(args.steps, 40))
    value, per_step, kind = run_cpu(c, cores, T_sample, steps, min(warm, 3))
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": steps, "warmup": min(warm, 3), "ms_per_step": per_step * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp16 rows, fp32 combine", "data": "synthetic",
        "config": config_json(c, 1, "n/a (host memory)"),
        "cpu_baseline": {
            "value": value, "unit": UNIT, "cores": cores, "kind": kind,
            "sample": f"{cores} host threads, each packing + combining its own {T_sample}-token slice of the "
                      f"{args.config} batch per step (reference moe::cpu_scatter from the unchanged source "
                      f"+ fp32 combine restatement)"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------ GPU arm -----

def gpu_arm(args):
    import torch
    import torch.distributed as dist
    import moe_b200 as mb

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    c = workload(args.config, rank)
    c["name"] = args.config
    T, K, E, d = c["T"], c["K"], c["E"], c["d"]
    TK = T * K
    tdtype = getattr(torch, c["dtype"])
    asgn_np, wts_np = routing.gen_routing(T, K, E, c["dist"], c["seed"])
    emb = routing.gen_rows(T, d, c["dtype"], c["seed"], device=dev)
    asgn = torch.from_numpy(asgn_np).to(dev)
    wts = torch.from_numpy(wts_np).to(dev)

    stream = torch.cuda.Stream(device=dev)
    warm = max(args.warmup, 3)
    flusher = L2Flush(dev)
    with torch.cuda.stream(stream):
        ws = mb.Workspace(T, K, E, device=dev, stream=stream)
        bufs = mb.pack(emb, asgn, wts, E, workspace=ws, stream=stream)
        out = torch.empty((T, d), dtype=tdtype, device=dev)

    if world > 1:
        import ep
        bounds = ep.expert_ranges(E, world)
        bounds_dev = torch.tensor(bounds, dtype=torch.long, device=dev)
        recv_buf = torch.empty((world * TK, d), dtype=tdtype, device=dev)
        back_buf = torch.empty((TK, d), dtype=tdtype, device=dev)

    def step(split=False):
        """One pass.  Returns CUDA events recorded on the launching stream at the
        step boundaries, plus one between pack and the rest when `split` (an
        event there costs the PDL overlap, so the headline loop omits it)."""
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(3 if split else 2)]
        evs[0].record(stream)
        mb.pack(emb, asgn, wts, E, workspace=ws, out=bufs, stream=stream)
        if split:
            evs[1].record(stream)
        y = bufs.packed
        if world > 1:
            starts = bufs.expert_start.long()
            send = (starts[bounds_dev[1:]] - starts[bounds_dev[:-1]]).to(torch.int64)
            recv = torch.empty_like(send)
            dist.all_to_all_single(recv, send)
            counts = torch.stack([send, recv]).cpu()  # host split sizes (one D2H, as the reference)
            s_list, r_list = counts[0].tolist(), counts[1].tolist()
            nrecv = sum(r_list)
            dist.all_to_all_single(recv_buf[:nrecv], bufs.packed, r_list, s_list)
            # identity expert on recv_buf[:nrecv]; combine back to the senders' packed order
            dist.all_to_all_single(back_buf, recv_buf[:nrecv], s_list, r_list)
            y = back_buf
        mb.unpermute(y, bufs.packed_weights, bufs.slot_pos, T, K, out=out, stream=stream)
        evs[-1].record(stream)
        return evs

    with torch.cuda.stream(stream):
        for i in range(warm):
            flusher(i)
            step()
        torch.cuda.synchronize(dev)
        assert ws.device_status(stream) == 0, "device-side condition during warm-up"
        # correctness gate before timing (identity expert closed form)
        ref = (wts.sum(dim=1, keepdim=True) * emb.float())
        torch.testing.assert_close(out.float(), ref, rtol=1e-3, atol=1e-3)

        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        rec = []
        with ClockSampler(local) as clk:
            for i in range(args.steps):
                flusher(i)
                rec.append(step())
            torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        # attribution loop: the same steps with an event between pack and the rest
        split = []
        for i in range(args.steps):
            flusher(i)
            split.append(step(split=True))
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()

    step_ms = [a.elapsed_time(b) for a, b in rec]
    pack_ms = [a.elapsed_time(b) for a, b, _ in split]
    rest_ms = [b.elapsed_time(cc) for _, b, cc in split]
    total_ms = sum(step_ms)
    if world > 1:
        t = torch.tensor([total_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())

    # e2e through the C ABI with pinned host buffers (N = 1 only)
    e2e = None
    if world == 1 and not args.no_e2e:
        e2e = e2e_leg(mb, c, emb, asgn_np, wts_np, ws, stream, dev, args.steps, warm)

    if rank == 0:
        b_pack, b_unperm = algorithmic_bytes(c)
        ms = total_ms / args.steps
        value = world * T * args.steps / (total_ms / 1e3)
        mean_pack = statistics.fmean(pack_ms)
        mean_rest = statistics.fmean(rest_ms)
        peak, peak_src = measured_peaks()
        if mean_rest >= mean_pack or world > 1:
            dom, dom_bytes, dom_ms = "unpermute_bulk_kernel", b_unperm, mean_rest
        else:
            dom, dom_bytes, dom_ms = "pack (route_scan_kernel + pack_rows_bulk_kernel)", b_pack, mean_pack
        if world > 1:
            dom, dom_bytes, dom_ms = "pack (route_scan_kernel + pack_rows_bulk_kernel)", b_pack, mean_pack
        achieved = dom_bytes / (dom_ms / 1e3) / 1e9
        traffic_key = "unpermute_kernel" if dom.startswith("unpermute") else "pack"
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": warm, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp16 rows (bitwise pack), fp32 combine accumulate",
            "data": "synthetic (seeded Gumbel top-K routing, N(0,1) rows)",
            "config": config_json(c, world, L2_NOTE),
            "hbm_gbs": (b_pack + b_unperm) / (ms / 1e3) / 1e9 if world == 1 else None,
            "stages_ms": {"pack": mean_pack, "unpermute" if world == 1 else "dispatch+combine+unpermute": mean_rest,
                          "note": "separate loop with an extra event between the stages (costs the "
                                  "PDL overlap); the headline step has events at its boundaries only"},
            "roofline": {
                "bound": "hbm", "kernel": dom, "achieved": achieved, "peak": peak, "unit": "GB/s",
                "frac": achieved / peak, "peak_source": f"{peak_src} (MEASURED_PEAKS.json hbm_gbs)"
                if peak_src == "measured" else "fallback 6.65 TB/s",
                "algorithmic_bytes_per_launch": dom_bytes,
                "traffic": committed_traffic(traffic_key, c["name"]),
            },
            "gpu_launches": 3 * args.steps,
            "kernels_per_step": ["route_scan_kernel", "pack_rows_bulk_kernel", "unpermute_bulk_kernel"],
            "clocks": clk.summary(),
        }
        if e2e is not None:
            line["e2e"] = e2e
        if world == 1 and not args.no_cpu_baseline:
            cv, per, kind = run_cpu(c, 1, c["T"], 5, 1, min_seconds=10.0)
            line["cpu_baseline"] = {
                "value": cv, "unit": UNIT, "cores": 1, "kind": kind,
                "sample": f"the full {c['name']} batch ({c['T']} tokens) packed by the reference's own "
                          f"moe::cpu_scatter (unchanged source, -O2) + the fp32 combine restatement, "
                          f"repeated for ~10 s ({per * 1e3:.1f} ms per batch) on 1 host thread of "
                          f"{host_cores()}"}
        print(json.dumps(line), flush=True)

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def e2e_leg(mb, c, emb_dev, asgn_np, wts_np, ws, stream, dev, steps, warm):
    """Same step through the public entry points, host buffers in and out."""
    import torch
    T, K, E, d = c["T"], c["K"], c["E"], c["d"]
    h_emb = emb_dev.cpu().pin_memory()
    h_asgn = torch.from_numpy(asgn_np).pin_memory()
    h_wts = torch.from_numpy(wts_np).pin_memory()
    h_out = torch.empty((T, d), dtype=emb_dev.dtype).pin_memory()
    d_emb = torch.empty_like(emb_dev)
    d_asgn = torch.empty((T, K), dtype=torch.int32, device=dev)
    d_wts = torch.empty((T, K), dtype=torch.float32, device=dev)
    d_out = torch.empty((T, d), dtype=emb_dev.dtype, device=dev)
    bufs = None
    flusher = L2Flush(dev)
    times = []
    with torch.cuda.stream(stream):
        for i in range(warm + steps):
            flusher(i)
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record(stream)
            d_emb.copy_(h_emb, non_blocking=True)
            d_asgn.copy_(h_asgn, non_blocking=True)
            d_wts.copy_(h_wts, non_blocking=True)
            bufs = mb.pack(d_emb, d_asgn, d_wts, E, workspace=ws, out=bufs, stream=stream)
            mb.unpermute(bufs.packed, bufs.packed_weights, bufs.slot_pos, T, K, out=d_out, stream=stream)
            h_out.copy_(d_out, non_blocking=True)
            b.record(stream)
            if i >= warm:
                times.append((a, b))
        torch.cuda.synchronize(dev)
    total = sum(a.elapsed_time(b) for a, b in times)
    h2d = T * d * 2 + T * K * 4 * 2
    d2h = T * d * 2
    return {"value": T * steps / (total / 1e3), "unit": UNIT, "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "ms_per_step": total / steps}


def main():
    args = parse()
    if args.impl == "reference":
        reference_arm(args)
    else:
        gpu_arm(args)


if __name__ == "__main__":
    main()
