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
          ranks' tokens / max-rank time.  The fused step is ONE library call
          per rank (moe_b200_ep_step, four kernels for the identity expert).

Prints ONE JSON line on rank 0.  `value` is device-timed (CUDA events on the
launching stream, created before the loop; inputs resident in HBM; L2 flushed
by a 256 MiB write + a 256 MiB read before every step); `e2e` is the same
metric through the C ABI with pinned host buffers and the host<->device
copies inside the timed region.  The default pack config also carries a
`layer` object: the full MoE layer (config c5: grouped SwiGLU experts) at the
same GPU count, the north-star "EP MoE layer us".  At N > 1 every rank checks
its fused-EP output bit for bit against the single-GPU path run on the same
batch before timing.  `clocks`: SM clock and clock-event reasons of every
GPU of the job, read through NVML every 2 ms during the timed region by a
separate sampling process (nvidia-smi -lms 200 when NVML is unavailable).
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
# NVLink: peer copy per direction measured on this pool's B200s (900 GB/s nominal)
NVLINK_GBS = 770.0


def parse(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--config", default="c2", choices=["c1", "c2", "c3", "c4", "c4u", "c5"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-layer", action="store_true",
                    help="pack configs: skip the c5 layer measurement that the line carries as `layer`")
    ap.add_argument("--no-c3", action="store_true",
                    help="N=1 default: skip the c3 (prefill-scale packing) measurement the line carries as `c3`")
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
    ap.add_argument("--_clock-child", dest="clock_child", default=None, help=argparse.SUPPRESS)
    return ap.parse_args(argv)


def workload(cfg_name, rank=0):
    base = "c4" if cfg_name == "c4u" else cfg_name
    c = dict(routing.CONFIGS[base])
    if cfg_name == "c4u":            # config 4's comparison run: the same shape, uniform routing
        c["dist"] = "uniform"
    c["name"] = cfg_name
    c["seed"] = c["seed"] + rank
    return c


def config_json(c, n, l2_note):
    xfer = {"fused": "peer-store exchange over NVLink", "nccl": "NCCL AllToAllv"}.get(c.get("ep", "fused"))
    n_pipe = 1 if xfer is None else n   # the CPU reference: one host, nothing to exchange
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


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f)
    except Exception:
        return None


def measured_peaks():
    p = _peaks()
    if p and "hbm_gbs" in p:
        return float(p["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def measured_tflops():
    p = _peaks()
    if p and "bf16_tflops_sustained" in p:
        return (float(p["bf16_tflops_sustained"]),
                "measured sustained bf16 (MEASURED_PEAKS.json bf16_tflops_sustained): the GEMMs run inside a "
                "millisecond-long layer step under the power cap")
    return 1400.0, "fallback 1.4 PFLOP/s sustained"


def committed_traffic(kernel, workload_name):
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            return json.load(f).get(f"{kernel}@{workload_name}")
    except Exception:
        return None


def stats_ms(xs):
    s = sorted(xs)
    return {"median": statistics.median(s), "p90": s[min(len(s) - 1, int(round(0.9 * (len(s) - 1))))],
            "max": s[-1], "min": s[0]}


# --------------------------------------------------------------- clocks ----

def clock_child(spec):
    """Runs in its own process: samples the SM clock and the clock-event
    reason bits of the given GPUs (NVML, by UUID or index) every 2 ms between
    a "go" and a "stop" line on stdin, then prints one JSON line.  Reading
    only: no clock, power or other setting is touched."""
    import select
    targets = json.loads(spec)
    try:
        import pynvml
        pynvml.nvmlInit()
        hs = []
        for t in targets:
            h = None
            if isinstance(t, str):
                for cand in (t, "GPU-" + t):
                    try:
                        h = pynvml.nvmlDeviceGetHandleByUUID(cand)
                        break
                    except Exception:
                        h = None
            if h is None:
                h = pynvml.nvmlDeviceGetHandleByIndex(int(t) if not isinstance(t, str) else 0)
            hs.append(h)
        get_reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
        smax = max(float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)) for h in hs)
    except Exception as e:  # noqa: BLE001
        print(json.dumps({"error": f"NVML unavailable: {e}"}), flush=True)
        return
    print("ready", flush=True)
    sys.stdin.readline()
    samples = []
    while True:
        for h in hs:
            try:
                samples.append((float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)), int(get_reasons(h))))
            except Exception:
                pass
        r, _, _ = select.select([sys.stdin], [], [], 0.002)
        if r:
            break
    print(json.dumps({"samples": samples, "smax": smax}), flush=True)
    try:
        pynvml.nvmlShutdown()
    except Exception:
        pass


class ClockSampler:
    """Samples the SM clock and clock-event (throttle) reasons of the job's
    GPUs while the timed region runs.  A separate process (clock_child) polls
    NVML every 2 ms, so the sampling neither holds this process's interpreter
    nor adds driver calls to the ranks' launch path; falls back to
    `nvidia-smi -lms 200` when NVML cannot be opened.  Only reads."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = (("hw_slowdown", "HwSlowdown", 0x8), ("hw_thermal_slowdown", "HwThermalSlowdown", 0x40),
               ("sw_thermal_slowdown", "SwThermalSlowdown", 0x20), ("sw_power_cap", "SwPowerCap", 0x4))

    def __init__(self, gpu_index, uuid=None, targets=None, indices=None):
        self.gpu = gpu_index
        self.targets = targets if targets is not None else [str(uuid) if uuid else gpu_index]
        self.indices = indices if indices is not None else [gpu_index]
        self.child = None
        self.proc = None
        self.lines = []
        self.samples = []            # (sm MHz, reason bit mask) from NVML
        self.smax = None

    def start(self):
        """Launch the sampling process (before warm-up: it takes a moment)."""
        try:
            self.child = subprocess.Popen([sys.executable, os.path.abspath(__file__), "--_clock-child",
                                           json.dumps(self.targets)], stdin=subprocess.PIPE,
                                          stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            first = self.child.stdout.readline().strip()
            if first != "ready":
                self.child.wait(timeout=10)
                self.child = None
        except Exception:
            self.child = None
        return self

    def __enter__(self):
        if self.child is None and self.proc is None:
            self.start()
        if self.child is not None:
            self.child.stdin.write("go\n")
            self.child.stdin.flush()
            return self
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", ",".join(str(i) for i in self.indices), f"--query-gpu={self.FIELDS}",
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
        if self.child is not None:
            try:
                self.child.stdin.write("stop\n")
                self.child.stdin.flush()
                out = json.loads(self.child.stdout.readline())
                self.samples = [tuple(s) for s in out.get("samples", [])]
                self.smax = out.get("smax")
                self.child.wait(timeout=10)
            except Exception:
                self.child.kill()
            self.child = None
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
                    "samples": len(self.samples), "gpus": len(self.targets),
                    "source": "NVML every 2 ms during the timed region, from a separate sampling process, all "
                              "GPUs of the job"}
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


class NullClock:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        pass


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


def make_events(n, stream):
    """n timing events, each recorded once so the CUDA event objects exist
    before any timed region (torch creates them lazily at the first record)."""
    import torch
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(n)]
    for e in evs:
        e.record(stream)
    return evs


# ----------------------------------------------------------- CPU legs -----

def _oracle():
    """The CPU checker package (oracle/): only the CPU legs of this file use it."""
    path = os.path.join(ROOT, "oracle")
    if path not in sys.path:
        sys.path.insert(0, path)
    import oracle
    return oracle


def cpu_inputs(c, T_sample):
    import torch
    asgn, wts = routing.gen_routing(c["T"], c["K"], c["E"], c["dist"], c["seed"])
    rows = routing.gen_rows(T_sample, c["d"], c["dtype"], c["seed"])
    emb = rows.view(torch.int16).numpy().view(np.uint16)
    return emb, np.ascontiguousarray(asgn[:T_sample]), np.ascontiguousarray(wts[:T_sample])


class CpuWorker:
    """One host thread's buffers for the CPU path: the reference's own
    moe::cpu_scatter (oracle/_ref, unchanged source) when built here, else the
    oracle restatement; then the oracle combine (the reference has no CPU
    combine).  ctypes drops the GIL, so threads run in parallel."""

    def __init__(self, emb, asgn, wts, E, dtype_code, slot_pos):
        oracle = _oracle()
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
        self.slot_pos = slot_pos
        self.out = np.zeros((T, d), np.uint16)
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
                                        p(np.empty(self.T * self.K, np.int32)))
        self.o.lib().oracle_combine(p(self.packed), p(self.pw), p(self.slot_pos), self.T, self.K, self.d,
                                    self.dt, p(self.out))


def run_cpu(c, threads, T_sample, steps, warmup, min_seconds=0.0):
    """Returns (tokens/s over all threads, seconds per step, kind, steps).
    With min_seconds, the step count grows until the timed work lasts that
    long.  Every thread packs + combines its own copy of the same batch."""
    oracle = _oracle()
    emb, asgn, wts = cpu_inputs(c, T_sample)
    dt = 0 if c["dtype"] == "float16" else 1
    slot_pos = oracle.scatter(emb, asgn, wts, c["E"])["slot_pos"]  # inverse of perm, for the combine
    workers = [CpuWorker(emb, asgn, wts, c["E"], dt, slot_pos) for _ in range(threads)]

    def parallel_step():
        ths = [threading.Thread(target=w.step) for w in workers]
        t0 = time.perf_counter()
        for th in ths:
            th.start()
        for th in ths:
            th.join()
        return time.perf_counter() - t0

    one = 0.0
    for _ in range(max(warmup, 1)):
        one = parallel_step()
    if min_seconds > 0:
        steps = max(steps, min(400, int(min_seconds / max(one, 1e-6)) + 1))
    times = [parallel_step() for _ in range(steps)]
    total = sum(times)
    return threads * T_sample * steps / total, total / steps, workers[0].kind, steps


def host_cores():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def reference_arm(args):
    """The reference's own CPU implementation of the path (moe::cpu_scatter,
    compiled unchanged, + the combine restatement) on every host thread, each
    thread packing and combining the FULL batch of the config per step, with
    the GPU arm's steps and warm-up."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    c = workload(args.config)
    c["ep"] = "host"
    c["placement"] = "n/a (every rank's tokens on the host cores)" if args.gpus > 1 else "n/a"
    if c.get("I"):
        print(json.dumps({"impl": "reference", "unavailable": "the reference has no CPU expert FFN; the CPU arm "
                          "covers the pack configs (c1-c4)"}), flush=True)
        return
    cores = host_cores()
    warm = max(args.warmup, 3)
    steps = max(1, args.steps)
    value, per_step, kind, steps = run_cpu(c, cores, c["T"], steps, warm)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": steps, "warmup": warm, "ms_per_step": per_step * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp16 rows, fp32 combine", "data": "synthetic",
        "config": config_json(c, args.gpus, "n/a (host memory)"),
        "cpu_baseline": {
            "value": value, "unit": UNIT, "cores": cores, "kind": kind,
            "sample": f"{cores} host threads, each packing + combining the full {c['T']}-token {args.config} batch "
                      f"per step (reference moe::cpu_scatter from the unchanged source + fp32 combine "
                      f"restatement)"},
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
        evs = make_events(2 * steps, stream)
        for i in range(steps):
            flusher(i)
            evs[2 * i].record(stream)
            mb.route(emb, rw, K, out=out, stream=stream)
            evs[2 * i + 1].record(stream)
        torch.cuda.synchronize(dev)
    assert mb.device_status(stream) == 0, "device-side condition in the router"
    us = statistics.median(evs[2 * i].elapsed_time(evs[2 * i + 1]) for i in range(steps)) * 1e3
    nbytes = T * d * 2 + T * K * 8 + (3 if emb.dtype == torch.bfloat16 else 2) * ((E + 15) // 16 * 16) * d * 2
    peak, _ = measured_peaks()
    gbs = nbytes / (us / 1e6) / 1e9
    return {"kernel": "route_kernel (gate GEMM + softmax + top-K)", "us": us, "tokens_per_s": T / (us / 1e6),
            "algorithmic_bytes": nbytes, "achieved_gbs": gbs, "peak_gbs": peak, "frac": gbs / peak,
            "traffic": committed_traffic("route_kernel", c["name"]),
            "note": "median device time per launch, L2 flushed before each; bytes = tokens read once + "
                    "outputs + the prepared gate weights once"}


class Job:
    """Rank / device / process-group facts shared by the measurements."""

    def __init__(self):
        import torch
        import torch.distributed as dist
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(self.local)
        self.dev = torch.device("cuda", self.local)
        self.dist = dist
        if self.world > 1:
            import datetime
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=self.dev)

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()

    def allreduce(self, values, op="max"):
        """Elementwise max (or sum) over ranks of a list of floats."""
        import torch
        if self.world == 1:
            return list(values)
        t = torch.tensor(values, dtype=torch.float64, device=self.dev)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX if op == "max" else self.dist.ReduceOp.SUM)
        return t.tolist()

    def gather_counts(self, expert_count, E):
        """[world, E] int64 numpy array of every rank's expert counts."""
        import torch
        if self.world == 1:
            return expert_count[:E].cpu().numpy().astype(np.int64)[None, :]
        allc = torch.empty((self.world, E), dtype=torch.int32, device=self.dev)
        self.dist.all_gather_into_tensor(allc.view(-1), expert_count[:E].contiguous())
        return allc.cpu().numpy().astype(np.int64)


def expert_weights(labels, orig_of, I, d, tdtype, dev):
    """Random-init SwiGLU experts ~N(0, 0.02), seeded by GLOBAL expert id so
    every rank count uses the same weights (apps/bench_prefill.cu:432-439):
    w_gate_up [n, 2I, d], w_down [n, d, I] for the given labels in order."""
    import torch
    n = len(labels)
    wgu = torch.empty((n, 2 * I, d), dtype=tdtype, device=dev)
    wdn = torch.empty((n, d, I), dtype=tdtype, device=dev)
    for j, lab in enumerate(labels):
        g = torch.Generator(device=dev)
        g.manual_seed(1000 + orig_of[lab])
        wgu[j] = (torch.randn((2 * I, d), generator=g, device=dev) * 0.02).to(tdtype)
        wdn[j] = (torch.randn((d, I), generator=g, device=dev) * 0.02).to(tdtype)
    return wgu, wdn


def run_config(args, job, cfg_name, clock, headline, e2e=True):
    """Measures one config at the job's GPU count.  Returns a dict of results
    (rank 0's view; every rank takes the same collective steps)."""
    import torch
    import moe_b200 as mb
    import ep

    world, rank, dev = job.world, job.rank, job.dev
    c = workload(cfg_name, rank)
    c["placement"] = args.placement if world > 1 else "n/a"
    c["ep"] = args.ep
    layer = "I" in c                       # c5: the full layer with SwiGLU experts
    gather = layer and world == 1 and args.gather
    if layer and world == 1:
        c["rows"] = ("gathered by the gate/up GEMM from the token rows (tile::gather4 by perm); pack writes "
                     "indices only" if gather else "packed copy")
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
        seed0 = routing.CONFIGS[cfg_name]["seed"]
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
    orig_of = {lab: e for e, lab in enumerate(label)}
    asgn = torch.from_numpy(asgn_np).to(dev)
    wts = torch.from_numpy(wts_np).to(dev)

    stream = torch.cuda.Stream(device=dev)
    warm = max(args.warmup, 3)
    steps = args.steps
    flusher = L2Flush(dev)
    bounds = ep.expert_ranges(E, world)
    fused = world > 1 and args.ep == "fused"
    # the most popular experts (routing.gen_routing: popularity falls with the
    # expert index), by their labels under the placement
    replicated = sorted(label[e] for e in range(min(args.replicate, E))) if fused else []
    fep = None
    if fused:
        with torch.cuda.stream(stream):
            fep = ep.FusedExpertParallel(E, K, d, T, tdtype, device=dev, timeout_ms=5000, replicated=replicated)
        local_labels = fep.local_experts
    else:
        local_labels = list(range(bounds[rank], bounds[rank + 1])) if world > 1 else list(range(E))
    with torch.cuda.stream(stream):
        ws = mb.Workspace(T, K, E, device=dev, stream=stream)
        bufs = mb.pack(emb, asgn, wts, E, workspace=ws, stream=stream, rows=not gather and not fused)
        out = torch.empty((T, d), dtype=tdtype, device=dev)
        I = c.get("I", 0)
        wgu = wdn = h_buf = y_buf = None
        if layer:
            wgu, wdn = expert_weights(local_labels, orig_of, I, d, tdtype, dev)
            cap = fep.recv_cap if fused else (world * TK if world > 1 else TK)
            h_buf = torch.empty((cap, I), dtype=tdtype, device=dev)
            if not fused:   # the fused down GEMM stores straight into the senders' back buffers
                y_buf = torch.empty((cap, d), dtype=tdtype, device=dev)
    epx = None
    if world > 1 and not fused:
        epx = ep.ExpertParallel(E, device=dev)
        recv_buf = torch.empty((world * TK, d), dtype=tdtype, device=dev)
        back_buf = torch.empty((TK, d), dtype=tdtype, device=dev)

    def enqueue(x_emb, x_asgn, x_wts, y_out):
        """One step through the public entry points, on `stream`."""
        if fused:
            fep.step(x_emb, x_asgn, x_wts, ws, bufs, y_out, wgu, wdn, h_buf, stream=stream)
            return
        mb.pack(x_emb, x_asgn, x_wts, E, workspace=ws, out=bufs, stream=stream)
        if world > 1:
            x_in, lay = epx.dispatch(bufs.packed, bufs.expert_count, recv_buf)
            seg_start, seg_expert = lay.seg_start, lay.seg_expert
        elif gather:
            x_in, seg_start, seg_expert = x_emb, bufs.expert_start, None
        else:
            x_in, seg_start, seg_expert = bufs.packed, bufs.expert_start, None
        if layer:
            n = TK if gather else x_in.shape[0]
            _, y = mb.grouped_swiglu(x_in, seg_start, wgu, wdn, seg_expert=seg_expert, h=h_buf[:n], y=y_buf[:n],
                                     stream=stream, row_token=bufs.perm if gather else None)
        else:
            y = x_in                                  # identity expert
        if world > 1:
            y = epx.combine(y, lay, back_buf)
        mb.unpermute(y, bufs.packed_weights, bufs.slot_pos, T, K, out=y_out, stream=stream)

    def split_step(evs):
        """The same step with events between the stages [start, pack(+dispatch)
        done, expert start, expert(+return) done, combine start, end] (an event
        between kernels costs the PDL overlap, so the headline loop does not
        split)."""
        evs[0].record(stream)
        if fused:
            fep.dispatch(emb, asgn, wts, ws, bufs, stream=stream)
            evs[1].record(stream)
            fep.receive(stream=stream)
            evs[2].record(stream)
            if layer:
                fep.ffn_return(wgu, wdn, h_buf, stream=stream)
            else:
                fep.return_identity(stream=stream)
            evs[3].record(stream)
            evs[4].record(stream)
            fep.combine(bufs.packed_weights, bufs.slot_pos, T, out, stream=stream)
            evs[5].record(stream)
            return
        mb.pack(emb, asgn, wts, E, workspace=ws, out=bufs, stream=stream)
        evs[1].record(stream)
        if world > 1:
            x_in, lay = epx.dispatch(bufs.packed, bufs.expert_count, recv_buf)
            seg_start, seg_expert = lay.seg_start, lay.seg_expert
        elif gather:
            x_in, seg_start, seg_expert = emb, bufs.expert_start, None
        else:
            x_in, seg_start, seg_expert = bufs.packed, bufs.expert_start, None
        evs[2].record(stream)
        if layer:
            n = TK if gather else x_in.shape[0]
            _, y = mb.grouped_swiglu(x_in, seg_start, wgu, wdn, seg_expert=seg_expert, h=h_buf[:n], y=y_buf[:n],
                                     stream=stream, row_token=bufs.perm if gather else None)
        else:
            y = x_in
        evs[3].record(stream)
        if world > 1:
            y = epx.combine(y, lay, back_buf)
        evs[4].record(stream)
        mb.unpermute(y, bufs.packed_weights, bufs.slot_pos, T, K, out=out, stream=stream)
        evs[5].record(stream)

    res = {"c": c, "T": T, "TK": TK, "layer": layer, "gather": gather, "fused": fused, "replicated": replicated,
           "bounds": bounds, "label": label}
    with torch.cuda.stream(stream):
        for i in range(warm):
            flusher(i)
            enqueue(emb, asgn, wts, out)
        torch.cuda.synchronize(dev)
        assert ws.device_status(stream) == 0, "device-side condition during warm-up"
        assert mb.device_status(stream) == 0, "device-side condition during warm-up"

        # ---- correctness gate before timing ----
        if world > 1:
            # bit-exact: every rank's expert-parallel output against the
            # single-GPU path (pack -> expert -> unpermute) on its own batch
            ref_bufs = mb.pack(emb, asgn, wts, E, stream=stream)
            if layer:
                all_labels = list(range(E))
                wgu_all, wdn_all = expert_weights(all_labels, orig_of, I, d, tdtype, dev)
                _, y_ref = mb.grouped_swiglu(ref_bufs.packed, ref_bufs.expert_start, wgu_all, wdn_all,
                                             stream=stream)
                del wgu_all, wdn_all
            else:
                y_ref = ref_bufs.packed
            ref_out = mb.unpermute(y_ref, ref_bufs.packed_weights, ref_bufs.slot_pos, T, K, stream=stream)
            torch.cuda.synchronize(dev)
            mism = int((out.view(torch.int16) != ref_out.view(torch.int16)).sum().item())
            del ref_bufs, y_ref, ref_out
            tot = job.allreduce([float(mism), float(mism > 0)], op="sum")
            res["parity"] = {"check": "bit-exact: every rank's expert-parallel output vs the single-GPU pack -> "
                                      + ("grouped SwiGLU" if layer else "identity") + " -> unpermute of the same "
                                      "batch on the same GPU", "mismatched_values": int(tot[0]),
                             "mismatched_ranks": int(tot[1]), "ok": tot[0] == 0}
            if tot[0] != 0:
                raise SystemExit(f"expert-parallel output differs from the single-GPU path: {res['parity']}")
        elif not layer:
            ref = (wts.sum(dim=1, keepdim=True) * emb.float())
            torch.testing.assert_close(out.float(), ref, rtol=1e-3, atol=1e-3)
            res["parity"] = {"check": "identity-expert closed form out = (sum_k w) * emb, rtol 1e-3 (the "
                                      "bit-exact oracle comparison runs in the -m gpu tests)", "ok": True}
        else:
            assert bool(torch.isfinite(out.float()).all()), "non-finite layer output"
            res["parity"] = {"check": "finite output (the kernel parity runs in the -m gpu tests)", "ok": True}

        # ---- timed loop: events at the step boundaries only ----
        evs = make_events(2 * steps, stream)
        split_evs = [make_events(6, stream) for _ in range(steps)]
        torch.cuda.synchronize(dev)
        job.barrier()
        torch.cuda.synchronize(dev)
        host_us = []
        with (clock if headline else NullClock()):
            for i in range(steps):
                flusher(i)
                t0 = time.perf_counter()
                evs[2 * i].record(stream)
                enqueue(emb, asgn, wts, out)
                evs[2 * i + 1].record(stream)
                host_us.append((time.perf_counter() - t0) * 1e6)
            torch.cuda.synchronize(dev)
        job.barrier()
        torch.cuda.synchronize(dev)
        # ---- attribution loop: the same steps with events between the stages ----
        for i in range(steps):
            flusher(i)
            split_step(split_evs[i])
        torch.cuda.synchronize(dev)
        job.barrier()
    assert ws.device_status(stream) == 0, "device-side condition during timing"
    assert mb.device_status(stream) == 0, "device-side condition during timing"

    step_ms = [evs[2 * i].elapsed_time(evs[2 * i + 1]) for i in range(steps)]
    st = stats_ms(step_ms)
    hs = stats_ms(host_us)
    sp = split_evs
    pack_ms = statistics.fmean(e[0].elapsed_time(e[1]) for e in sp)
    mid_ms = statistics.fmean(e[1].elapsed_time(e[4]) for e in sp)       # dispatch + expert + combine
    recv_ms = statistics.fmean(e[1].elapsed_time(e[2]) for e in sp)
    expert_ms = statistics.fmean(e[2].elapsed_time(e[3]) for e in sp)
    unperm_ms = statistics.fmean(e[4].elapsed_time(e[5]) for e in sp)
    agg = job.allreduce([sum(step_ms), st["median"], st["p90"], st["max"], hs["median"], hs["max"], pack_ms,
                         mid_ms, recv_ms, expert_ms, unperm_ms])
    (total_ms, med, p90, mx, h_med, h_max, pack_ms, mid_ms, recv_ms, expert_ms, unperm_ms) = agg
    # L2 norm of the last step's output over all tokens of all ranks, the
    # reference's multi-GPU consistency check (apps/bench_prefill.cu:955-972)
    sumsq = job.allreduce([float(out.float().square().sum(dtype=torch.float64).item())], op="sum")[0]
    res.update(total_ms=total_ms, ms=total_ms / steps, warm=warm, steps=steps,
               step_stats_ms={"median": med, "p90": p90, "max": mx,
                              "note": "per-step device time (events at step boundaries); each figure is the max "
                                      "over ranks"},
               host_enqueue_us={"median": h_med, "max": h_max,
                                "note": "host time to enqueue one step (library calls + 2 event records), max "
                                        "over ranks"},
               stages={"pack": pack_ms, "mid": mid_ms, "receive": recv_ms, "expert": expert_ms,
                       "unpermute": unperm_ms},
               out_l2=sumsq ** 0.5)
    counts = job.gather_counts(bufs.expert_count, E)
    res["counts"] = counts

    # the router (gate GEMM + softmax + top-K) on the same tokens, timed alone
    # with the same L2 flush: the step before the packing path in the
    # reference's bench_e2e pipeline (apps/bench_e2e.cu:231-246)
    if headline and world == 1 and not layer and not args.no_router:
        res["router"] = router_leg(mb, c, emb, stream, dev, flusher, steps, warm)

    if e2e and not args.no_e2e:
        res["e2e"] = e2e_leg(job, c, emb, asgn_np, wts_np, enqueue, stream, steps, warm, layer)
    if fep is not None:
        fep.close()
    return res


def e2e_leg(job, c, emb_dev, asgn_np, wts_np, enqueue, stream, steps, warm, layer):
    """The same step through the public entry points, host buffers in and out.
    Every step copies its inputs H2D from pinned host memory and its result
    D2H; consecutive steps are pipelined the way a serving loop runs them:
    the H2D of step i+1 (copy stream) overlaps step i's compute and the D2H of
    step i-1 (second copy stream) -- PCIe is full duplex -- with two sets of
    device input/output buffers, and L2 is flushed on the compute stream
    before every step.  Time = first H2D to last D2H, max over ranks."""
    import torch
    dev = job.dev
    T, K, d = c["T"], c["K"], c["d"]
    h_emb = emb_dev.cpu().pin_memory()
    h_asgn = torch.from_numpy(asgn_np).pin_memory()
    h_wts = torch.from_numpy(wts_np).pin_memory()
    h_out = [torch.empty((T, d), dtype=emb_dev.dtype).pin_memory() for _ in range(2)]
    d_emb = [torch.empty_like(emb_dev) for _ in range(2)]
    d_asgn = [torch.empty((T, K), dtype=torch.int32, device=dev) for _ in range(2)]
    d_wts = [torch.empty((T, K), dtype=torch.float32, device=dev) for _ in range(2)]
    d_out = [torch.empty((T, d), dtype=emb_dev.dtype, device=dev) for _ in range(2)]
    s_in, s_out = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    flusher = L2Flush(dev)
    ev = lambda: torch.cuda.Event(enable_timing=False)  # noqa: E731
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
            enqueue(d_emb[k], d_asgn[k], d_wts[k], d_out[k])
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
    t1.record(s_out)
    torch.cuda.synchronize(dev)
    job.barrier()
    t0.record(s_in)
    for i in range(warm, warm + steps):
        run(i)
    s_out.wait_event(out_done[(warm + steps - 1) % 2])
    t1.record(s_out)
    torch.cuda.synchronize(dev)
    total = job.allreduce([t0.elapsed_time(t1)])[0]
    job.barrier()
    if not layer:
        # the result of the last step arrived intact
        ref = (torch.from_numpy(wts_np).sum(dim=1, keepdim=True) * h_emb.float())
        torch.testing.assert_close(h_out[(warm + steps - 1) % 2].float(), ref, rtol=1e-3, atol=1e-3)
    h2d = T * d * 2 + T * K * 4 * 2
    d2h = T * d * 2
    ms = total / steps
    return {"value": ms * 1e3 if layer else job.world * T * steps / (total / 1e3),
            "unit": "us" if layer else UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "ms_per_step": ms,
            "note": "through the C ABI (" + ("moe_b200_ep_step" if job.world > 1 and c.get("ep") == "fused"
                                             else "moe_b200_pack / grouped FFN / moe_b200_unpermute")
                    + "); per rank every step copies its inputs H2D from pinned memory and its output D2H; step "
                      "i+1's H2D overlaps step i's compute and step i-1's D2H on separate copy streams "
                      "(double-buffered device inputs/outputs); L2 flushed before every step; max over ranks"}


def kernels_of(res, world):
    layer, fused, gather = res["layer"], res["fused"], res["gather"]
    if fused:
        expert = (["ep_receive_kernel", "grouped_gemm_kernel<SwiGLU>",
                   "grouped_gemm_kernel<store, peer scatter, + back-flag signal>"] if layer
                  else ["ep_return_identity_kernel (+ data-flag wait, back-flag signal)"])
        return ["route_scan_kernel (+ count publish)", "ep_pack_dispatch_kernel"] + expert + \
            ["unpermute_bulk_kernel (+ back-flag wait)"]
    if gather:
        return ["route_scan_kernel", "pack_index_kernel", "grouped_gemm_kernel<SwiGLU, gathered rows>",
                "grouped_gemm_kernel<store>", "unpermute_bulk_kernel"]
    k = ["route_scan_kernel", "pack_rows_bulk_kernel", "unpermute_bulk_kernel"]
    if layer:
        k[2:2] = ["grouped_gemm_kernel<SwiGLU>", "grouped_gemm_kernel<store>"]
    if world > 1:
        k.append("ep_layout_kernel")
    return k


def exchange_bytes(res, world):
    """Per-rank rows that cross NVLink in the dispatch (the return moves the
    same rows back): sender r -> rank g for every non-replicated expert that g
    owns, g != r.  The survey's EP byte model."""
    counts, bounds, c = res["counts"], res["bounds"], res["c"]
    hot = set(res["replicated"])
    E, d = c["E"], c["d"]
    owner = np.zeros(E, np.int64)
    for g in range(world):
        owner[bounds[g]:bounds[g + 1]] = g
    remote = np.array([e not in hot for e in range(E)])
    send = [int(sum(counts[r][e] for e in range(E) if remote[e] and owner[e] != r)) * d * 2 for r in range(world)]
    recv = [int(sum(counts[s][e] for s in range(world) if s != r for e in range(E) if remote[e] and owner[e] == r))
            * d * 2 for r in range(world)]
    return send, recv


def layer_summary(res, world):
    c = res["c"]
    TK, d, I = res["TK"], c["d"], c["I"]
    tf_peak, tf_src = measured_tflops()
    flops = 6 * TK * d * I
    expert_ms = res["stages"]["expert"]
    achieved = flops / (expert_ms / 1e3) / 1e12
    return {"metric": METRIC_LAYER, "value": res["ms"] * 1e3, "unit": "us", "higher_is_better": False,
            "n_gpus": world, "steps": res["steps"], "warmup": res["warm"],
            "workload": config_json(c, world, L2_NOTE)["workload"] + f", I={I}, T split over {world} GPU(s)",
            "ffn_ms": expert_ms, "ffn_tflops": achieved, "ffn_frac": achieved / tf_peak, "ffn_peak_tflops": tf_peak,
            "ffn_peak_source": tf_src, "algorithmic_flops_per_rank": flops,
            "tokens_per_s": world * res["T"] * res["steps"] / (res["total_ms"] / 1e3),
            "checksum": {"output_l2": res["out_l2"],
                         "note": "L2 norm of the layer output over the whole batch (all ranks); every rank holds a "
                                 "slice of one global batch, so it is the same for every N"},
            "parity": res["parity"], "step_stats_ms": res["step_stats_ms"],
            "stages_ms": {"pack+dispatch": res["stages"]["pack"], "ffn(+return)": expert_ms,
                          "unpermute": res["stages"]["unpermute"]},
            **({"e2e": res["e2e"]} if "e2e" in res else {})}


def gpu_arm(args):
    import torch
    job = Job()
    world, rank = job.world, job.rank
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    # one sampling process on rank 0 for every GPU of the job
    uuid = str(getattr(torch.cuda.get_device_properties(job.dev), "uuid", "") or job.local)
    targets = [uuid]
    if world > 1:
        targets = [None] * world
        job.dist.all_gather_object(targets, uuid)
    clock = ClockSampler(job.local, targets=targets, indices=list(range(world))) if rank == 0 else NullClock()
    if rank == 0:
        clock.start()

    res = run_config(args, job, args.config, clock, headline=True)
    lay = None
    if not res["layer"] and not args.no_layer:
        torch.cuda.empty_cache()
        lay = run_config(args, job, "c5", NullClock(), headline=False)
    big = None
    if args.config == "c2" and world == 1 and not args.no_c3:
        torch.cuda.empty_cache()
        big = run_config(args, job, "c3", NullClock(), headline=False, e2e=False)

    if rank == 0:
        c = res["c"]
        ms = res["total_ms"] / args.steps
        layer = res["layer"]
        b_pack, b_unperm = algorithmic_bytes(c)
        peak_hbm, src_hbm = measured_peaks()
        kernels = kernels_of(res, world)
        stg = res["stages"]
        line = {
            "metric": METRIC_LAYER if layer else METRIC,
            "unit": "us" if layer else UNIT,
            "value": ms * 1e3 if layer else world * res["T"] * args.steps / (res["total_ms"] / 1e3),
            "n_gpus": world, "steps": args.steps, "warmup": res["warm"], "ms_per_step": ms,
            "higher_is_better": not layer, "scaling": "strong" if layer else "weak",
            "vs_baseline": None,
            "dtype": ("bf16 rows and weights, fp32 accumulate" if layer
                      else "fp16 rows (bitwise pack), fp32 combine accumulate"),
            "data": "synthetic (seeded Gumbel top-K routing, N(0,1) rows" +
                    (", N(0,0.02) random-init experts)" if layer else ")"),
            "config": config_json(c, world, L2_NOTE),
            "step_stats_ms": res["step_stats_ms"],
            "host_enqueue_us": res["host_enqueue_us"],
            "stages_ms": {"pack" + ("+dispatch" if world > 1 else ""): stg["pack"],
                          ("dispatch+ffn+combine" if world > 1 else "ffn") if layer else
                          ("receive+return" if world > 1 else "identity"): stg["mid"],
                          "unpermute": stg["unpermute"],
                          "note": "max over ranks of the per-rank means, from a separate loop with events "
                                  "between the stages (costs the PDL overlap); the headline step has events "
                                  "at its boundaries only"},
            "gpu_launches": len(kernels) * args.steps,
            "kernels_per_step": kernels,
            "clocks": clock.summary(),
            "parity": res["parity"],
            "checksum": {"output_l2": res["out_l2"],
                         "note": ("L2 norm of the layer output over the whole batch (all ranks); every rank "
                                  "holds a slice of one global batch, so it is the same for every N")
                         if layer else ("L2 norm of the output over all ranks' tokens (each rank its own "
                                        "seeded batch, so it grows with N)")},
        }
        if layer:
            ls = layer_summary(res, world)
            line["tokens_per_s"] = ls["tokens_per_s"]
            line["ffn_ms"] = ls["ffn_ms"]
            line["roofline"] = {
                "bound": "tensor", "kernel": "grouped_gemm_kernel (SwiGLU GEMM + down GEMM)",
                "achieved": ls["ffn_tflops"], "peak": ls["ffn_peak_tflops"], "unit": "TFLOP/s",
                "frac": ls["ffn_frac"], "peak_source": ls["ffn_peak_source"],
                "algorithmic_flops_per_launch": ls["algorithmic_flops_per_rank"],
                "traffic": committed_traffic("grouped_ffn", c["name"]),
            }
        elif world == 1:
            line["hbm_gbs"] = (b_pack + b_unperm) / (ms / 1e3) / 1e9
            if stg["unpermute"] >= stg["pack"]:
                dom, dom_bytes, dom_ms, key = "unpermute_bulk_kernel", b_unperm, stg["unpermute"], "unpermute_kernel"
            else:
                dom, dom_bytes, dom_ms, key = ("pack (route_scan_kernel + pack_rows_bulk_kernel)", b_pack,
                                               stg["pack"], "pack")
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
            send, recv = exchange_bytes(res, world)
            worst = max(max(send), max(recv))
            if res["fused"]:
                t_disp = stg["pack"]              # route_scan + dispatch, max over ranks
                t_ret = stg["expert"]             # identity return (or FFN + return), max over ranks
            else:                                 # NCCL: both AllToAllv (+ counts, D2H) in one stage
                t_disp = t_ret = stg["mid"] / 2
            gbs = worst / (t_disp / 1e3) / 1e9
            line["ep"] = {
                "experts_per_rank": [res["bounds"][g + 1] - res["bounds"][g] for g in range(world)],
                "replicated": (f"{len(res['replicated'])} most popular experts have a copy on every rank "
                               "(their rows stay local)") if res["replicated"] else "none",
                "placement": args.placement + (" (experts dealt over the ranks in serpentine order of popularity)"
                                               if args.placement == "balanced" else ""),
                "exchange": ("fused: pack stores rows into the owners' receive buffers over NVLink, the expert "
                             "stores them back into the senders' buffers; epoch flags in peer memory, no "
                             "collective library and no host sync on the data path; one library call per step")
                if res["fused"] else "NCCL all_gather (counts) + 2 x all_to_all_single (rows)",
                "remote_send_bytes_per_rank": send, "remote_recv_bytes_per_rank": recv,
                "dispatch_ms": t_disp, "return_ms": t_ret if not layer else None,
                "return_gbs": (worst / (t_ret / 1e3) / 1e9) if not layer else None,
            }
            if not layer:
                line["roofline"] = {
                    "bound": "nvlink",
                    "kernel": ("ep_pack_dispatch_kernel (+ route_scan_kernel before it)" if res["fused"] else
                               "NCCL all_to_all_single (half of the dispatch + combine stage, which also holds "
                               "the count all-gather and the D2H of the split sizes)"),
                    "achieved": gbs, "peak": NVLINK_GBS, "unit": "GB/s", "frac": gbs / NVLINK_GBS,
                    "peak_source": "measured peer copy per direction on this pool's B200s (profiling recipe); "
                                   "900 GB/s nominal",
                    "algorithmic_bytes_per_launch": worst,
                    "note": "bytes = the busiest rank's remote rows in its busier direction (max over ranks of "
                            "max(sent, received)); time = the pack+dispatch stage, max over ranks",
                    "traffic": None,
                }
        if "e2e" in res:
            line["e2e"] = res["e2e"]
        if "router" in res:
            line["router"] = res["router"]
        if lay is not None:
            line["layer"] = layer_summary(lay, world)
        if big is not None:
            b3p, b3u = algorithmic_bytes(big["c"])
            ms3 = big["ms"]
            line["c3"] = {
                "metric": METRIC, "unit": UNIT, "value": big["T"] * big["steps"] / (big["total_ms"] / 1e3),
                "ms_per_step": ms3, "workload": config_json(big["c"], 1, L2_NOTE)["workload"],
                "hbm_gbs": (b3p + b3u) / (ms3 / 1e3) / 1e9, "frac": (b3p + b3u) / (ms3 / 1e3) / 1e9 / peak_hbm,
                "stages_ms": {"pack": big["stages"]["pack"], "unpermute": big["stages"]["unpermute"]},
                "algorithmic_bytes_per_step": b3p + b3u, "parity": big["parity"],
                "note": "prefill-scale packing (BASELINE config 3), same step and timing as the headline"}
        if world == 1 and not args.no_cpu_baseline and not layer:
            cv, per, kind, n = run_cpu(c, 1, c["T"], 5, 1, min_seconds=10.0)
            line["cpu_baseline"] = {
                "value": cv, "unit": UNIT, "cores": 1, "kind": kind,
                "sample": f"the full {c['name']} batch ({c['T']} tokens) packed by the reference's own "
                          f"moe::cpu_scatter (unchanged source, -O2) + the fp32 combine restatement, "
                          f"{n} batches (~10 s, {per * 1e3:.1f} ms per batch) on 1 host thread of "
                          f"{host_cores()}"}
        print(json.dumps(line), flush=True)

    job.barrier()
    if world > 1:
        job.dist.destroy_process_group()


def main():
    args = parse()
    if args.clock_child is not None:
        clock_child(args.clock_child)
        return
    if args.impl == "reference":
        reference_arm(args)
    else:
        gpu_arm(args)


if __name__ == "__main__":
    main()
