"""bench.py end to end on one GPU, every workload at reduced sizes: the run
exits 0 and prints one JSON line with the contract's keys."""
import json
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("args", [
    ["--workload", "config4", "--layers", "2", "--steps", "3", "--warmup", "3", "--no-cpu-baseline"],
    ["--workload", "config3", "--experts", "96", "--tokens", "2048", "--steps", "2", "--warmup", "3",
     "--no-cpu-baseline"],
    ["--workload", "config4", "--format", "ternary106", "--layers", "2", "--steps", "3", "--warmup", "3"],
    ["--workload", "expert", "--format", "mxfp4", "--pool", "8", "--steps", "3", "--warmup", "3",
     "--cpu-seconds", "1"],
    ["--workload", "expert", "--format", "ternary106", "--pool", "8", "--steps", "3", "--warmup", "3",
     "--no-cpu-baseline"],
    ["--workload", "compress", "--pool", "2", "--steps", "2", "--warmup", "3", "--no-cpu-baseline"],
], ids=["config4", "config3", "config4-ternary106", "expert-mxfp4", "expert-ternary106", "compress"])
def test_bench_line(args):
    r = subprocess.run([sys.executable, "bench.py", *args], cwd=ROOT, capture_output=True, text=True,
                       timeout=900)
    assert r.returncode == 0, r.stderr[-3000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
              "dtype", "config", "roofline", "e2e", "gpu_launches", "clocks"):
        assert k in line, k
    assert line["value"] > 0 and line["gpu_launches"] > 0
    assert 0 < line["roofline"]["frac"] < 2
