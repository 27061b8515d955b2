"""The C++ layer harness (15618-final_b200/apps/bench_layer.cu) runs router ->
pack -> grouped SwiGLU FFN -> unpermute through the C ABI alone and checks the
outputs on the host (routing invariants, the cpu_scatter packing contract,
the inverse permutation, 4 tokens of layer output against an fp64 host
evaluation).  Here it runs on small shapes in both 16-bit types."""
import json
import os
import subprocess

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "15618-final_b200", "_build", "bench_layer")


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
@pytest.mark.parametrize("T,d,E,K,I", [(1000, 256, 16, 4, 128), (333, 512, 60, 2, 64)])
def test_bench_layer_checks_pass(cuda, dtype, T, d, E, K, I):
    if not os.path.exists(BIN):
        subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "15618-final_b200"), "apps"], check=True,
                       timeout=600)
    r = subprocess.run([BIN, "--T", str(T), "--d", str(d), "--E", str(E), "--K", str(K), "--I", str(I),
                        "--dtype", dtype, "--iters", "2", "--warmup", "1"],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["checks"] == "pass" and line["layer_ms"] > 0
