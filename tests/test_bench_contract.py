"""The benchmark's JSON contract, checked on the CPU through the reference
arm (`bench.py --impl reference`, the reference's own cpu_scatter + the
combine restatement on the host cores): one JSON line with the keys the
harness reads, at N = 1 and, under torchrun with two CPU ranks, only
rank 0 printing."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

KEYS = {"impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
        "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"}


def run(args, env=None):
    r = subprocess.run([sys.executable] + args, cwd=ROOT, capture_output=True, text=True, timeout=600,
                       env=env)
    assert r.returncode == 0, r.stderr[-2000:]
    return [ln for ln in r.stdout.splitlines() if ln.startswith("{")]


def test_reference_arm_line():
    lines = run(["bench.py", "--impl", "reference", "--steps", "1", "--warmup", "3"])
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert KEYS <= set(d)
    assert d["impl"] == "reference" and d["n_gpus"] == 1 and d["warmup"] >= 3
    assert d["value"] > 0 and d["unit"] == "tokens/s" and d["higher_is_better"] is True
    assert d["config"]["workload"].startswith("c2")
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and cb["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}


def _free_port():
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_reference_arm_prints_on_rank_zero_only():
    env = dict(os.environ, MASTER_ADDR="127.0.0.1")
    lines = run(["-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2", "--master-addr",
                 "127.0.0.1", "--master-port", str(_free_port()), "bench.py", "--impl", "reference", "--gpus", "2",
                 "--steps", "1", "--warmup", "3"], env=env)
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["n_gpus"] == 2 and d["config"]["parallelism"] == "ep2"


def test_clock_summary_names_reasons_from_nvml_bits():
    """ClockSampler.summary() on injected samples (no GPU, no NVML calls):
    median SM clock, and every clock-event reason bit seen during the region."""
    sys.path.insert(0, ROOT)
    import pynvml
    import bench
    c = bench.ClockSampler(0)
    c.smax = 1965.0
    cap, slow = pynvml.nvmlClocksEventReasonSwPowerCap, pynvml.nvmlClocksEventReasonHwSlowdown
    c.samples = [(1965.0, 0), (1800.0, cap), (1965.0, 0), (1500.0, cap | slow)]
    s = c.summary()
    assert s["sm_mhz"] == 1882.5 and s["sm_min_mhz"] == 1500.0 and s["samples"] == 4
    assert s["reasons"] == ["hw_slowdown", "sw_power_cap"]
    c.samples = [(1965.0, pynvml.nvmlClocksEventReasonGpuIdle)]
    assert c.summary()["reasons"] == []
    # nvidia-smi fallback lines
    c = bench.ClockSampler(0)
    c.lines = ["0, 1965, 1965, 700.1, 0x0, Not Active, Not Active, Not Active, Active",
               "0, 1950, 1965, 710.0, 0x0, Not Active, Not Active, Not Active, Not Active"]
    s = c.summary()
    assert s["sm_mhz"] == 1957.5 and s["sm_max_mhz"] == 1965.0 and s["reasons"] == ["sw_power_cap"]


def test_exchange_byte_model_and_step_stats():
    """bench.exchange_bytes: rows a rank sends to / receives from other ranks
    (non-replicated experts owned elsewhere), the survey's EP byte model, on
    a hand-checked 2-rank case; bench.stats_ms on a known list."""
    sys.path.insert(0, ROOT)
    import numpy as np
    import bench
    # E = 4 experts, ranks own [0, 2) and [2, 4); expert 1 replicated
    counts = np.array([[5, 7, 2, 1],     # rank 0's rows per expert
                       [3, 4, 6, 8]])    # rank 1's
    res = {"counts": counts, "bounds": [0, 2, 4], "replicated": [1], "c": {"E": 4, "d": 8}}
    send, recv = bench.exchange_bytes(res, 2)
    row = 8 * 2
    assert send == [(2 + 1) * row, 3 * row]      # rank 0 -> experts 2, 3; rank 1 -> expert 0 (1 is local)
    assert recv == [3 * row, (2 + 1) * row]
    s = bench.stats_ms([5.0, 1.0, 3.0, 2.0, 4.0])
    assert s["median"] == 3.0 and s["max"] == 5.0 and s["min"] == 1.0 and s["p90"] == 5.0
