"""Benchmark of the MoE token packing + weighted unpermute path.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--config c2]

One step = one pass of the hot path over one batch:
  N = 1   pack (route_scan + pack_rows) -> identity expert -> unpermute, on the
          single-B200 workload (config c2: T=8192, d=2048 fp16, E=60, K=4,
          Zipf s=1.2 routing).
  N > 1   (torchrun, one rank per GPU) each rank packs its own T=8192 tokens
          and stores the packed rows straight into the expert-owning ranks'
          receive buffers over NVLink (CUDA IPC peer memory; `--ep nccl`
          selects the AllToAllv variant), applies the identity expert, returns
          the rows the same way and unpermutes: weak scaling, value = all
          ranks' tokens / max-rank time.

Prints ONE JSON line on rank 0.  `value` is device-timed (CUDA events on the
launching stream, inputs resident in HBM, L2 flushed by a 256 MiB write + a
256 MiB read before every step); `e2e` is the same metric through the C ABI with pinned host
buffers and the host<->device copies inside the timed region.  `clocks`: the
SM clock and clock-event reasons read through NVML every 2 ms during the
timed region (nvidia-smi -lms 200 when NVML is unavailable).
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
METRIC_LAYER = "EP MoE layer us"
UNIT = "tokens/s"
FALLBACK_HBM_GBS = 6650.0


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--config", default="c2", choices=["c1", "c2", "c3", "c4", "c5"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--placement", default="balanced", choices=["balanced", "contiguous"],
                    help="N>1 expert placement: popularity dealt round-robin over ranks (default) or the "
                         "reference's contiguous ranges")
    ap.add_argument("--gather", action="store_true",
                    help="N=1 layer (c5): the gate/up GEMM gathers the token rows (tile::gather4 by perm) and the "
                         "pack writes indices only (measured slower on B200; default: packed rows)")
    ap.add_argument("--no-router", action="store_true",
                    help="skip the separate router timing (N=1 pack configs)")
    ap.add_argument("--replicate", type=int, default=8,
                    help="N>1 fused EP: the R most popular experts get a copy on every rank, so their rows "
                         "stay local (0 = the reference's pure partition)")
    ap.add_argument("--ep", default="fused", choices=["fused", "nccl"],
                    help="N>1 exchange: fused peer-store kernels (default) or NCCL AllToAllv")
    return ap.parse_args()


def workload(cfg_name, rank=0):
    c = dict(routing.CONFIGS[cfg_name])
    c["seed"] = c["seed"] + rank
    return c


def config_json(c, n, l2_note):
    xfer = {"fused": "peer-store exchange over NVLink", "nccl": "NCCL AllToAllv"}.get(c.get("ep", "fused"))
    if xfer is None:            # the CPU reference: one host, nothing to exchange
        n_pipe = 1
    else:
        n_pipe = n
    return {
        "workload": f"{c['name']}: T={c['T']} per GPU, d={c['d']} {c['dtype']}, E={c['E']}, "
                    f"K={c['K']}, {c['dist']} routing" + (" s=1.2" if c["dist"] == "zipf" else ""),
        "T_per_gpu": c["T"], "d": c["d"], "E": c["E"], "K": c["K"], "routing": c["dist"],
        "expert": f"SwiGLU FFN, I={c['I']}" if c.get("I") else "identity",
        "pipeline": ("pack -> " + ("" if n_pipe == 1 else xfer + " -> ")
                     + ("grouped SwiGLU FFN" if c.get("I") else "identity")
                     + ("" if n_pipe == 1 else " -> " + xfer) + " -> unpermute"),
        "parallelism": f"ep{n}" if n > 1 else "single-gpu",
        **({"rows": c["rows"]} if "rows" in c else {}),
        "placement": c.get("placement", "n/a"),
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


def measured_tflops():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return (float(p["bf16_tflops_sustained"]),
                "measured sustained bf16 (MEASURED_PEAKS.json bf16_tflops_sustained): the GEMMs run inside a "
                "millisecond-long layer step under the power cap")
    except Exception:
        return 1400.0, "fallback 1.4 PFLOP/s sustained"


def committed_traffic(kernel, workload_name):
    path = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(path) as f:
            return json.load(f).get(f"{kernel}@{workload_name}")
    except Exception:
        return None


# --------------------------------------------------------------- clocks ----

class ClockSampler:
    """Samples one GPU's SM clock and clock-event (throttle) reasons while the
    timed region runs.  Reads NVML (the library nvidia-smi queries) every 2 ms
    from a thread, so even a timed region of a few milliseconds gets samples;
    falls back to `nvidia-smi -lms 200` when NVML cannot be opened.  Only
    reads: no clock, power or other setting is touched."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = (("hw_slowdown", "HwSlowdown", 0x8), ("hw_thermal_slowdown", "HwThermalSlowdown", 0x40),
               ("sw_thermal_slowdown", "SwThermalSlowdown", 0x20), ("sw_power_cap", "SwPowerCap", 0x4))

    def __init__(self, gpu_index, uuid=None):
        self.gpu = gpu_index
        self.uuid = uuid
        self.proc = None
        self.nvml = None
        self.lines = []
        self.samples = []            # (sm MHz, reason bit mask) from NVML
        self.smax = None

    def _open_nvml(self):
        import pynvml
        pynvml.nvmlInit()
        h = None
        if self.uuid:
            u = str(self.uuid)
            for cand in (u, "GPU-" + u):
                try:
                    h = pynvml.nvmlDeviceGetHandleByUUID(cand)
                    break
                except Exception:
                    h = None
        if h is None:
            h = pynvml.nvmlDeviceGetHandleByIndex(self.gpu)
        get_reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
        self.smax = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
        self.nvml = (pynvml, h, get_reasons)

    def _poll_nvml(self):
        pynvml, h, get_reasons = self.nvml
        while not self.stop.is_set():
            try:
                self.samples.append((float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)),
                                     int(get_reasons(h))))
            except Exception:
                pass
            self.stop.wait(0.002)

    def __enter__(self):
        self.stop = threading.Event()
        try:
            self._open_nvml()
            self.thread = threading.Thread(target=self._poll_nvml, daemon=True)
            self.thread.start()
            return self
        except Exception:
            self.nvml = None
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
        if self.nvml:
            self.stop.set()
            self.thread.join(timeout=5)
            try:
                self.nvml[0].nvmlShutdown()
            except Exception:
                pass
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if self.samples:
            import pynvml
            reasons = set()
            for name, suffix, bit in self.REASONS:
                mask = getattr(pynvml, "nvmlClocksEventReason" + suffix, bit)
                if any(r & mask for _, r in self.samples):
                    reasons.add(name)
            return {"sm_mhz": statistics.median(c for c, _ in self.samples), "sm_max_mhz": self.smax,
                    "sm_min_mhz": min(c for c, _ in self.samples), "reasons": sorted(reasons),
                    "samples": len(self.samples), "source": "NVML, every 2 ms during the timed region"}
        if not self.lines:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["clock sampling unavailable"]}
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
                "reasons": sorted(reasons), "samples": len(sm), "source": "nvidia-smi -lms 200"}


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
    c["ep"] = "host"
    c["placement"] = "n/a (every rank's tokens on the host cores)" if args.gpus > 1 else "n/a"
    cores = host_cores()
    T_sample = min(c["T"], 2048)
    warm = max(args.warmup, 3)
    steps = max(1, min(args.steps, 40))
    value, per_step, kind = run_cpu(c, cores, T_sample, steps, min(warm, 3))
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": steps, "warmup": min(warm, 3), "ms_per_step": per_step * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp16 rows, fp32 combine", "data": "synthetic",
        "config": config_json(c, args.gpus, "n/a (host memory)"),
        "cpu_baseline": {
            "value": value, "unit": UNIT, "cores": cores, "kind": kind,
            "sample": f"{cores} host threads, each packing + combining its own {T_sample}-token slice of the "
                      f"{args.config} batch per step (reference moe::cpu_scatter from the unchanged source "
                      f"+ fp32 combine restatement)"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------ GPU arm -----

def router_leg(mb, c, emb, stream, dev, flusher, steps, warm):
    """Times moe_b200_route on the workload's tokens: random gate weights
    U(-0.05, 0.05) [d, E] fp32 (the reference's fill_random_float,
    include/moe/fp16_host.hpp:32-39), L2 flushed before every launch."""
    import torch
    T, K, E, d = c["T"], c["K"], c["E"], c["d"]
    g = torch.Generator(device=dev)
    g.manual_seed(42)
    w_gate = (torch.rand((d, E), generator=g, device=dev) - 0.5) * 0.1
    with torch.cuda.stream(stream):
        rw = mb.RouterWeights(w_gate, emb.dtype, stream=stream)
        out = (torch.empty((T, K), dtype=torch.int32, device=dev),
               torch.empty((T, K), dtype=torch.float32, device=dev))
        for i in range(warm):
            flusher(i)
            mb.route(emb, rw, K, out=out, stream=stream)
        evs = []
        for i in range(steps):
            flusher(i)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            mb.route(emb, rw, K, out=out, stream=stream)
            b.record(stream)
            evs.append((a, b))
        torch.cuda.synchronize(dev)
    assert mb.device_status(stream) == 0, "device-side condition in the router"
    us = statistics.median(a.elapsed_time(b) for a, b in evs) * 1e3
    nbytes = T * d * 2 + T * K * 8 + (3 if emb.dtype == torch.bfloat16 else 2) * ((E + 15) // 16 * 16) * d * 2
    peak, _ = measured_peaks()
    gbs = nbytes / (us / 1e6) / 1e9
    return {"kernel": "route_kernel (gate GEMM + softmax + top-K)", "us": us, "tokens_per_s": T / (us / 1e6),
            "algorithmic_bytes": nbytes, "achieved_gbs": gbs, "peak_gbs": peak, "frac": gbs / peak,
            "traffic": committed_traffic("route_kernel", c["name"]),
            "note": "median device time per launch, L2 flushed before each; bytes = tokens read once + "
                    "outputs + the prepared gate weights once"}


def gpu_arm(args):
    import torch
    import torch.distributed as dist
    import moe_b200 as mb
    import ep

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
    c["placement"] = args.placement if world > 1 else "n/a"
    c["ep"] = args.ep
    if "I" in c and world == 1:
        c["rows"] = ("gathered by the gate/up GEMM from the token rows (tile::gather4 by perm); pack writes "
                     "indices only" if args.gather else "packed copy")
    layer = "I" in c                       # c5: the full layer with SwiGLU experts
    T_glob = c["T"]
    if layer:
        # the layer's T tokens are split over the ranks (apps/bench_prefill.cu:341)
        if c["T"] % world:
            raise SystemExit(f"T={c['T']} not divisible by {world} ranks")
        c["T"] = c["T"] // world
    T, K, E, d = c["T"], c["K"], c["E"], c["d"]
    TK = T * K
    tdtype = getattr(torch, c["dtype"])
    if layer:
        # every rank takes its slice of ONE global batch, so the layer's
        # outputs (and the checksum below) are the same for every N
        seed0 = routing.CONFIGS[args.config]["seed"]
        a_g, w_g = routing.gen_routing(T_glob, K, E, c["dist"], seed0)
        asgn_np = np.ascontiguousarray(a_g[rank * T:(rank + 1) * T])
        wts_np = np.ascontiguousarray(w_g[rank * T:(rank + 1) * T])
        emb = routing.gen_rows(T_glob, d, c["dtype"], seed0, device=dev)[rank * T:(rank + 1) * T].contiguous()
    else:
        asgn_np, wts_np = routing.gen_routing(T, K, E, c["dist"], c["seed"])
        emb = routing.gen_rows(T, d, c["dtype"], c["seed"], device=dev)
    label = list(range(E))
    if world > 1 and args.placement == "balanced":
        label = ep.balanced_labels(E, world)
        asgn_np = np.asarray(label, dtype=np.int32)[asgn_np]
    orig_of = {l: e for e, l in enumerate(label)}
    asgn = torch.from_numpy(asgn_np).to(dev)
    wts = torch.from_numpy(wts_np).to(dev)

    stream = torch.cuda.Stream(device=dev)
    warm = max(args.warmup, 3)
    flusher = L2Flush(dev)
    bounds = ep.expert_ranges(E, world)
    lo, hi = bounds[rank], bounds[rank + 1]
    fused = world > 1 and args.ep == "fused"
    # the most popular experts (routing.gen_routing: popularity falls with the
    # expert index), by their labels under the placement
    replicated = sorted(label[e] for e in range(min(args.replicate, E))) if fused else []
    if fused:
        with torch.cuda.stream(stream):
            fep = ep.FusedExpertParallel(E, K, d, T, tdtype, device=dev, timeout_ms=5000, replicated=replicated)
        local_labels = fep.local_experts
    else:
        local_labels = list(range(lo, hi))
    # --gather: the gate/up GEMM gathers the token rows itself (TMA
    # tile::gather4 by perm), so the pack writes indices only
    gather = layer and world == 1 and args.gather
    with torch.cuda.stream(stream):
        ws = mb.Workspace(T, K, E, device=dev, stream=stream)
        bufs = mb.pack(emb, asgn, wts, E, workspace=ws, stream=stream, rows=not gather)
        out = torch.empty((T, d), dtype=tdtype, device=dev)
        if layer:
            I = c["I"]
            # random-init experts ~N(0, 0.02), seeded by GLOBAL expert id so every
            # rank count uses the same weights (apps/bench_prefill.cu:432-439)
            nl = len(local_labels)
            wgu = torch.empty((nl, 2 * I, d), dtype=tdtype, device=dev)
            wdn = torch.empty((nl, d, I), dtype=tdtype, device=dev)
            for j, lab in enumerate(local_labels):
                g = torch.Generator(device=dev)
                g.manual_seed(1000 + orig_of[lab])
                wgu[j] = (torch.randn((2 * I, d), generator=g, device=dev) * 0.02).to(tdtype)
                wdn[j] = (torch.randn((d, I), generator=g, device=dev) * 0.02).to(tdtype)
            cap = world * TK if world > 1 else TK
            h_buf = torch.empty((cap, I), dtype=tdtype, device=dev)
            y_buf = torch.empty((cap, d), dtype=tdtype, device=dev)
    if world > 1 and not fused:
        epx = ep.ExpertParallel(E, device=dev)
        recv_buf = torch.empty((world * TK, d), dtype=tdtype, device=dev)
        back_buf = torch.empty((TK, d), dtype=tdtype, device=dev)
    if fused and layer:
        with torch.cuda.stream(stream):
            h_buf = torch.empty((fep.recv_cap, c["I"]), dtype=tdtype, device=dev)

    def step(split=False):
        """One pass.  Returns CUDA events recorded on the launching stream: the
        step boundaries only, or with `split` six boundaries [start, pack done,
        expert start, expert done, combine done, end] (an event between
        kernels costs the PDL overlap, so the headline loop does not split)."""
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(6 if split else 2)]
        mark = (lambda i: evs[i].record(stream)) if split else (lambda i: None)
        evs[0].record(stream)
        if fused:
            fep.dispatch(emb, asgn, wts, ws, bufs, stream=stream)
            mark(1)
            fep.receive(stream=stream)
            mark(2)
            if layer:
                fep.ffn_return(wgu, wdn, h_buf, stream=stream)
            else:
                fep.return_identity(stream=stream)
            mark(3)
            mark(4)
            fep.combine(bufs.packed_weights, bufs.slot_pos, T, out, stream=stream)
            evs[-1].record(stream)
            return evs
        mb.pack(emb, asgn, wts, E, workspace=ws, out=bufs, stream=stream)
        mark(1)
        if world > 1:
            x_in, lay = epx.dispatch(bufs.packed, bufs.expert_count, recv_buf)
            seg_start, seg_expert = lay.seg_start, lay.seg_expert
        elif gather:
            x_in, seg_start, seg_expert = emb, bufs.expert_start, None
        else:
            x_in, seg_start, seg_expert = bufs.packed, bufs.expert_start, None
        mark(2)
        if layer:
            n = TK if gather else x_in.shape[0]
            _, y = mb.grouped_swiglu(x_in, seg_start, wgu, wdn, seg_expert=seg_expert,
                                     h=h_buf[:n], y=y_buf[:n], stream=stream,
                                     row_token=bufs.perm if gather else None)
        else:
            y = x_in                                  # identity expert
        mark(3)
        if world > 1:
            y = epx.combine(y, lay, back_buf)
        mark(4)
        mb.unpermute(y, bufs.packed_weights, bufs.slot_pos, T, K, out=out, stream=stream)
        evs[-1].record(stream)
        return evs

    with torch.cuda.stream(stream):
        for i in range(warm):
            flusher(i)
            step()
        torch.cuda.synchronize(dev)
        assert ws.device_status(stream) == 0, "device-side condition during warm-up"
        assert mb.device_status(stream) == 0, "device-side condition during warm-up"
        if not layer:
            # correctness gate before timing (identity expert closed form)
            ref = (wts.sum(dim=1, keepdim=True) * emb.float())
            torch.testing.assert_close(out.float(), ref, rtol=1e-3, atol=1e-3)
        else:
            assert bool(torch.isfinite(out.float()).all()), "non-finite layer output"

        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        rec = []
        with ClockSampler(local, getattr(torch.cuda.get_device_properties(dev), "uuid", None)) as clk:
            for i in range(args.steps):
                flusher(i)
                rec.append(step())
            torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        # attribution loop: the same steps with events between the stages
        split = []
        for i in range(args.steps):
            flusher(i)
            split.append(step(split=True))
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()

    step_ms = [a.elapsed_time(b) for a, b in rec]
    pack_ms = [e[0].elapsed_time(e[1]) for e in split]
    mid_ms = [e[1].elapsed_time(e[4]) for e in split]       # dispatch + expert + combine
    expert_ms = [e[2].elapsed_time(e[3]) for e in split]
    unperm_ms = [e[4].elapsed_time(e[5]) for e in split]
    total_ms = sum(step_ms)
    stage = torch.tensor([statistics.fmean(pack_ms), statistics.fmean(mid_ms), statistics.fmean(expert_ms),
                          statistics.fmean(unperm_ms)], dtype=torch.float64, device=dev)
    # L2 norm of the last step's output over all tokens of all ranks, the
    # reference's multi-GPU consistency check (apps/bench_prefill.cu:955-972)
    sumsq = out.float().square().sum(dtype=torch.float64).reshape(1)
    if world > 1:
        t = torch.tensor([total_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
        dist.all_reduce(stage, op=dist.ReduceOp.MAX)
        dist.all_reduce(sumsq, op=dist.ReduceOp.SUM)
    out_l2 = float(sumsq.item()) ** 0.5
    mean_pack, mean_mid, mean_expert, mean_unperm = stage.tolist()

    # The router (gate GEMM + softmax + top-K) on the same tokens, timed alone
    # with the same L2 flush: the step before the packing path in the
    # reference's bench_e2e pipeline (apps/bench_e2e.cu:231-246).
    router = None
    if world == 1 and not layer and not args.no_router:
        router = router_leg(mb, c, emb, stream, dev, flusher, args.steps, warm)

    # e2e through the C ABI with pinned host buffers: pipelined across steps
    # for the single-GPU pack path; elsewhere (expert parallel, the layer)
    # every step is H2D -> step -> D2H on the step's stream, max over ranks
    e2e = None
    if world == 1 and not args.no_e2e and not layer:
        e2e = e2e_leg(mb, c, emb, asgn_np, wts_np, ws, stream, dev, args.steps, warm)
    elif not args.no_e2e:
        h_emb = emb.cpu().pin_memory()
        h_asgn = asgn.cpu().pin_memory()
        h_wts = wts.cpu().pin_memory()
        h_out = torch.empty(out.shape, dtype=out.dtype).pin_memory()
        spans = []
        with torch.cuda.stream(stream):
            for i in range(warm + args.steps):
                flusher(i)
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                emb.copy_(h_emb, non_blocking=True)
                asgn.copy_(h_asgn, non_blocking=True)
                wts.copy_(h_wts, non_blocking=True)
                step()
                h_out.copy_(out, non_blocking=True)
                b.record(stream)
                if i >= warm:
                    spans.append((a, b))
            torch.cuda.synchronize(dev)
        e2e_ms = torch.tensor([sum(x.elapsed_time(y) for x, y in spans)], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
        ms_e2e = float(e2e_ms.item()) / args.steps
        h2d = T * d * 2 + T * K * 8
        e2e = {"value": ms_e2e * 1e3 if layer else world * T / (ms_e2e / 1e3),
               "unit": "us" if layer else UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": T * d * 2,
               "ms_per_step": ms_e2e,
               "note": "per rank, every step: inputs H2D from pinned memory, the step, the output D2H, on "
                       "one stream; max over ranks"}

    if rank == 0:
        ms = total_ms / args.steps
        b_pack, b_unperm = algorithmic_bytes(c)
        peak_hbm, src_hbm = measured_peaks()
        kernels = ["route_scan_kernel", "pack_rows_bulk_kernel", "unpermute_bulk_kernel"]
        if layer:
            kernels[2:2] = ["grouped_gemm_kernel<SwiGLU>", "grouped_gemm_kernel<store>"]
        if gather:
            kernels = ["route_scan_kernel", "pack_index_kernel", "grouped_gemm_kernel<SwiGLU, gathered rows>",
                       "grouped_gemm_kernel<store>", "unpermute_bulk_kernel"]
        if fused:
            kernels = ["route_scan_kernel", "ep_publish_kernel", "ep_pack_dispatch_kernel", "ep_receive_kernel"] + \
                (["grouped_gemm_kernel<SwiGLU>", "grouped_gemm_kernel<store, peer scatter>"] if layer
                 else ["ep_return_identity_kernel"]) + ["ep_signal_kernel", "ep_wait_kernel",
                                                        "unpermute_bulk_kernel"]
        line = {
            "metric": METRIC_LAYER if layer else METRIC,
            "unit": "us" if layer else UNIT,
            "value": ms * 1e3 if layer else world * T * args.steps / (total_ms / 1e3),
            "n_gpus": world, "steps": args.steps, "warmup": warm, "ms_per_step": ms,
            "higher_is_better": not layer, "scaling": "strong" if layer else "weak",
            "vs_baseline": None,
            "dtype": ("bf16 rows and weights, fp32 accumulate" if layer
                      else "fp16 rows (bitwise pack), fp32 combine accumulate"),
            "data": "synthetic (seeded Gumbel top-K routing, N(0,1) rows" +
                    (", N(0,0.02) random-init experts)" if layer else ")"),
            "config": config_json(c, world, L2_NOTE),
            "stages_ms": {"pack": mean_pack,
                          ("dispatch+ffn+combine" if world > 1 else "ffn") if layer else
                          ("dispatch+combine" if world > 1 else "identity"): mean_mid,
                          "unpermute": mean_unperm,
                          "note": "max over ranks of the per-rank means, from a separate loop with events "
                                  "between the stages (costs the PDL overlap); the headline step has events "
                                  "at its boundaries only"},
            "gpu_launches": len(kernels) * args.steps + (args.steps if world > 1 and not fused else 0),
            "kernels_per_step": kernels + (["ep_layout_kernel"] if world > 1 and not fused else []),
            "clocks": clk.summary(),
            "checksum": {"output_l2": out_l2,
                         "note": ("L2 norm of the layer output over the whole batch (all ranks); every rank "
                                  "holds a slice of one global batch, so it is the same for every N")
                         if layer else ("L2 norm of the output over all ranks' tokens (each rank its own "
                                        "seeded batch, so it grows with N)")},
        }
        if layer:
            I = c["I"]
            flops = 6 * world * TK * d * I  # all ranks' FFN work; per rank ~ 6 * TK * d * I
            tf_peak, tf_src = measured_tflops()
            achieved = 6 * TK * d * I / (mean_expert / 1e3) / 1e12
            line["tokens_per_s"] = world * T * args.steps / (total_ms / 1e3)
            line["roofline"] = {
                "bound": "tensor", "kernel": "grouped_gemm_kernel (SwiGLU GEMM + down GEMM)",
                "achieved": achieved, "peak": tf_peak, "unit": "TFLOP/s", "frac": achieved / tf_peak,
                "peak_source": tf_src, "algorithmic_flops_per_launch": 6 * TK * d * I,
                "traffic": committed_traffic("grouped_ffn", c["name"]),
            }
            line["ffn_ms"] = mean_expert
        else:
            if world == 1:
                line["hbm_gbs"] = (b_pack + b_unperm) / (ms / 1e3) / 1e9
            if mean_unperm >= mean_pack and world == 1:
                dom, dom_bytes, dom_ms, key = "unpermute_bulk_kernel", b_unperm, mean_unperm, "unpermute_kernel"
            else:
                dom, dom_bytes, dom_ms, key = ("pack (route_scan_kernel + pack_rows_bulk_kernel)", b_pack,
                                               mean_pack, "pack")
            achieved = dom_bytes / (dom_ms / 1e3) / 1e9
            line["roofline"] = {
                "bound": "hbm", "kernel": dom, "achieved": achieved, "peak": peak_hbm, "unit": "GB/s",
                "frac": achieved / peak_hbm,
                "peak_source": (f"{src_hbm} (MEASURED_PEAKS.json hbm_gbs)" if src_hbm == "measured"
                                else "fallback 6.65 TB/s"),
                "algorithmic_bytes_per_launch": dom_bytes,
                "traffic": committed_traffic(key, c["name"]),
            }
        if world > 1:
            line["ep"] = {"experts_per_rank": [bounds[g + 1] - bounds[g] for g in range(world)],
                          "replicated": (f"{len(replicated)} most popular experts have a copy on every rank "
                                         "(their rows stay local)") if replicated else "none",
                          "placement": args.placement + (" (expert e -> rank e % N by popularity rank)"
                                                         if args.placement == "balanced" else ""),
                          "exchange": ("fused: pack stores rows into the owners' receive buffers over NVLink, "
                                       "the expert stores them back into the senders' buffers; epoch flags in "
                                       "peer memory, no collective library and no host sync on the data path")
                          if fused else "NCCL all_gather (counts) + 2 x all_to_all_single (rows)"}
        if e2e is not None:
            line["e2e"] = e2e
        if router is not None:
            line["router"] = router
        if world == 1 and not args.no_cpu_baseline and not layer:
            cv, per, kind = run_cpu(c, 1, c["T"], 5, 1, min_seconds=10.0)
            line["cpu_baseline"] = {
                "value": cv, "unit": UNIT, "cores": 1, "kind": kind,
                "sample": f"the full {c['name']} batch ({c['T']} tokens) packed by the reference's own "
                          f"moe::cpu_scatter (unchanged source, -O2) + the fp32 combine restatement, "
                          f"repeated for ~10 s ({per * 1e3:.1f} ms per batch) on 1 host thread of "
                          f"{host_cores()}"}
        print(json.dumps(line), flush=True)

    if fused:
        fep.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def e2e_leg(mb, c, emb_dev, asgn_np, wts_np, ws, stream, dev, steps, warm):
    """Same step through the public entry points, host buffers in and out.
    Every step copies its inputs H2D from pinned host memory and its result
    D2H; consecutive steps are pipelined the way a serving loop runs them:
    the H2D of step i+1 (copy stream) overlaps the D2H of step i (second copy
    stream) -- PCIe is full duplex -- with two sets of device buffers, and L2
    is flushed on the compute stream before every pack.  Throughput = all
    steps over the time from the first H2D to the last D2H."""
    import torch
    T, K, E, d = c["T"], c["K"], c["E"], c["d"]
    h_emb = emb_dev.cpu().pin_memory()
    h_asgn = torch.from_numpy(asgn_np).pin_memory()
    h_wts = torch.from_numpy(wts_np).pin_memory()
    h_out = [torch.empty((T, d), dtype=emb_dev.dtype).pin_memory() for _ in range(2)]
    d_emb = [torch.empty_like(emb_dev) for _ in range(2)]
    d_asgn = [torch.empty((T, K), dtype=torch.int32, device=dev) for _ in range(2)]
    d_wts = [torch.empty((T, K), dtype=torch.float32, device=dev) for _ in range(2)]
    d_out = [torch.empty((T, d), dtype=emb_dev.dtype, device=dev) for _ in range(2)]
    wss = [ws, mb.Workspace(T, K, E, device=dev, stream=stream)]
    bufs = [None, None]
    s_in, s_out = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    flusher = L2Flush(dev)
    ev = lambda: torch.cuda.Event(enable_timing=False)
    in_ready, comp_done, out_done = [ev(), ev()], [ev(), ev()], [ev(), ev()]
    started = [False, False]

    def run(i):
        k = i % 2
        with torch.cuda.stream(s_in):
            if started[k]:
                s_in.wait_event(comp_done[k])       # step i-2 no longer reads these inputs
            d_emb[k].copy_(h_emb, non_blocking=True)
            d_asgn[k].copy_(h_asgn, non_blocking=True)
            d_wts[k].copy_(h_wts, non_blocking=True)
            in_ready[k].record(s_in)
        with torch.cuda.stream(stream):
            stream.wait_event(in_ready[k])
            if started[k]:
                stream.wait_event(out_done[k])      # step i-2's result has left d_out[k]
            flusher(i)
            bufs[k] = mb.pack(d_emb[k], d_asgn[k], d_wts[k], E, workspace=wss[k], out=bufs[k], stream=stream)
            mb.unpermute(bufs[k].packed, bufs[k].packed_weights, bufs[k].slot_pos, T, K, out=d_out[k],
                         stream=stream)
            comp_done[k].record(stream)
        with torch.cuda.stream(s_out):
            s_out.wait_event(comp_done[k])
            h_out[k].copy_(d_out[k], non_blocking=True)
            out_done[k].record(s_out)
        started[k] = True

    for i in range(warm):
        run(i)
    torch.cuda.synchronize(dev)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(s_in)
    for i in range(warm, warm + steps):
        run(i)
    s_out.wait_event(out_done[(warm + steps - 1) % 2])
    t1.record(s_out)
    torch.cuda.synchronize(dev)
    total = t0.elapsed_time(t1)
    # the result of the last step arrived intact
    ref = (torch.from_numpy(wts_np).sum(dim=1, keepdim=True) * h_emb.float())
    torch.testing.assert_close(h_out[(warm + steps - 1) % 2].float(), ref, rtol=1e-3, atol=1e-3)
    h2d = T * d * 2 + T * K * 4 * 2
    d2h = T * d * 2
    return {"value": T * steps / (total / 1e3), "unit": UNIT, "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "ms_per_step": total / steps,
            "note": "through moe_b200_pack / moe_b200_unpermute; every step copies its inputs H2D from pinned "
                    "memory and its output D2H; step i+1's H2D overlaps step i's D2H on separate copy streams "
                    "(double-buffered device buffers); L2 flushed before every pack"}


def main():
    args = parse()
    if args.impl == "reference":
        reference_arm(args)
    else:
        gpu_arm(args)


if __name__ == "__main__":
    main()
