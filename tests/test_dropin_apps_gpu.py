"""The reference's own applications, compiled unchanged and linked against
libmoe_b200 (`make -C oracle ref-apps`: moe::make_scatter comes from this
library's C++ IScatter shim, the reference strategies from their unchanged
sources), run on a GPU with strategy "b200":

  - apps/verify.cu: its mini test (:110-161) and the full run on a .npy
    workload (:166-263), both gated by verify_scatter_outputs;
  - apps/bench_scatter.cu: its one-shot correctness gate (:187-213);
  - apps/bench_e2e.cu: the mini layer (:331-371) and a full layer run;
  - with 2 or more GPUs, apps/bench_ep.cu and apps/bench_prefill.cu; for the
    latter the reference's own multi-GPU consistency check (the L2 norm of
    the combined rows, :955-972) must be identical with the b200 strategy and
    the reference's csort strategy.

Skipped where the reference-built binaries are absent (they are built where
the reference tree exists and travel with the repository)."""
import os
import re
import subprocess

import numpy as np
import pytest
import torch

import routing
from conftest import ROOT

pytestmark = pytest.mark.gpu

REF = os.path.join(ROOT, "oracle", "_ref")


def app(name):
    path = os.path.join(REF, name)
    if not os.path.exists(path):
        pytest.skip(f"{name} not built (make -C oracle ref-apps)")
    return path


def write_workload(d, prefix, T, E, K=4, dim=2048, dist="zipf", seed=0, ranks=1):
    """<prefix>_{embeddings,assignments,weights}.npy as the reference's apps
    read them: fp16 rows, int32 assignments, fp32 weights; with ranks > 1 the
    rank batches (seed + r) are stacked, T rows each."""
    embs, asgns, wtss = [], [], []
    for r in range(ranks):
        a, w = routing.gen_routing(T, K, E, dist, seed + r)
        x = routing.gen_rows(T, dim, "float16", seed + r)
        embs.append(x.view(torch.int16).numpy().view(np.float16))
        asgns.append(a)
        wtss.append(w)
    np.save(os.path.join(d, f"{prefix}_embeddings.npy"), np.concatenate(embs))
    np.save(os.path.join(d, f"{prefix}_assignments.npy"), np.concatenate(asgns))
    np.save(os.path.join(d, f"{prefix}_weights.npy"), np.concatenate(wtss))


def run(args, timeout=600):
    r = subprocess.run(args, capture_output=True, text=True, timeout=timeout)
    out = r.stdout + r.stderr
    assert r.returncode == 0, out[-3000:]
    return out


def test_verify_mini_and_full(cuda, tmp_path):
    exe = app("verify_b200")
    write_workload(tmp_path, "syn", 2048, 60)
    out = run([exe, "syn", "60", str(tmp_path), "b200"])
    assert "b200:             PASS" in out
    assert "b200 invariants: PASS" in out
    assert "ALL PASS" in out


def test_bench_scatter_correctness_gate(cuda, tmp_path):
    exe = app("bench_scatter_b200")
    write_workload(tmp_path, "syn", 8192, 60)
    out = run([exe, "--prefix=syn", "--E=60", f"--data-dir={tmp_path}", "--strategy=b200", "--warmup=2",
               "--iters=5", "--min-total-ms=0"])
    assert "correctness: PASS" in out


def test_bench_e2e_mini_and_full(cuda, tmp_path):
    exe = app("bench_e2e_b200")
    write_workload(tmp_path, "syn", 1024, 60, dim=512)
    out = run([exe, "syn", "60", str(tmp_path), "b200"])
    assert "Mini-test" in out
    assert "packing frac" in out


def test_bench_ep_two_gpus(cuda, tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 or more GPUs")
    exe = app("bench_ep_b200")
    write_workload(tmp_path, "syn", 4096, 64, dim=1024)
    out = run([exe, "--prefix=syn", f"--data-dir={tmp_path}", "--strategy=b200", "--n-gpus=2", "--E=64"],
              timeout=300)
    assert "total:" in out


def test_bench_prefill_checksum_matches_reference_strategy(cuda, tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 or more GPUs")
    exe = app("bench_prefill_b200")
    write_workload(tmp_path, "c4", 2048, 64, dim=512, ranks=2)
    l2 = {}
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    for st in ("csort", "b200"):
        r = subprocess.run([exe, "--prefix=c4", f"--data-dir={tmp_path}", f"--strategy={st}", "--n-gpus=2",
                            "--E=64", "--repeats=3", "--warmup=1"], capture_output=True, text=True, timeout=300,
                           env=env)
        assert r.returncode == 0, (r.stdout + r.stderr)[-3000:]
        m = re.search(r"L2 = ([0-9.]+)", r.stdout)
        assert m, r.stdout[-2000:]
        l2[st] = m.group(1)
    assert l2["b200"] == l2["csort"], l2
