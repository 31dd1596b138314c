"""bench.py pieces that run without a GPU: the reference arm's JSON line and
the workload-matched CPU samples."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("workload", ["ragged", "huge-pair", "dense", "embed128"])
def test_reference_arm_line(workload):
    out = subprocess.run(
        [sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--workload",
         workload, "--steps", "1", "--warmup", "0"],
        capture_output=True, text=True, timeout=600, cwd=ROOT,
        env={**os.environ, "OMP_NUM_THREADS": "2"})
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
                "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["value"] > 0
    assert line["e2e"]["h2d_bytes_per_step"] == 0
    assert line["cpu_baseline"]["kind"] == "port"
    # the reference arm describes the same workload as ours
    sys.path.insert(0, ROOT)
    import bench
    assert line["config"]["workload"] == bench.WORKLOADS[workload].describe(1)["workload"]
    assert line["scaling"] == bench.WORKLOADS[workload].scaling


def test_cpu_units_count_terms():
    sys.path.insert(0, ROOT)
    import bench
    run, label = next(bench.cpu_units("huge-pair"))
    assert run(1) == 256.0 * (262144 + 262144)
    run, label = next(bench.cpu_units("ragged"))
    x, y = bench.ragged_graph(0)
    n, m = x.shape[0], y.shape[0]
    assert run(1) == float(n * n + m * m + n * m)
