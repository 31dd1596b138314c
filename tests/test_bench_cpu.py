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
    # identical config dicts in both arms (the workload and its term counts)
    assert line["config"] == json.loads(json.dumps(bench.WORKLOADS[workload].describe(1)))
    assert line["config"]["full_terms_per_step"] > 0
    assert line["scaling"] == "strong"
    assert "oracle" in line["cpu_baseline"]["what"]


def test_cpu_units_count_terms():
    sys.path.insert(0, ROOT)
    import bench
    run, label = next(bench.cpu_units("huge-pair"))
    assert run(1) == 256.0 * (262144 + 262144)
    run, label = next(bench.cpu_units("ragged"))
    x, y = bench.ragged_graph(0)
    n, m = x.shape[0], y.shape[0]
    assert run(1) == float(n * n + m * m + n * m)


def test_strong_scaling_shares_cover_the_batch():
    """The LPT shares of the 4096-graph batch at 1, 2, 4 and 8 ranks add up to
    the configured term counts (what the multi-GPU line checks at run time)."""
    sys.path.insert(0, ROOT)
    import numpy as np
    import bench
    from rapidalign_b200.shard import lpt_partition
    cfg = bench.RaggedWorkload.describe(1)
    sizes = bench.ragged_sizes(range(cfg["graphs"]))
    cost = sizes[:, 0] ** 2 + sizes[:, 1] ** 2 + sizes[:, 0] * sizes[:, 1]
    for world in (1, 2, 4, 8):
        assert bench.RaggedWorkload.describe(world) == cfg
        full = 0.0
        for part in lpt_partition(cost, world):
            f, _ = bench.term_counts(sizes[part, 0], sizes[part, 1])
            full += f
        assert abs(full - cfg["full_terms_per_step"]) <= 1e-9 * full
    assert bench.RaggedWorkload.describe(4, "weak")["graphs"] == 4 * cfg["graphs"]


@pytest.mark.parametrize("workload", ["ragged", "embed128", "dense", "huge-pair"])
def test_reference_gpu_arm_without_a_gpu(workload):
    """The reference's own CUDA kernels are timed only on a GPU and only for
    the D=3 ragged batch; otherwise the arm prints why, and exits 0."""
    out = subprocess.run(
        [sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference-gpu",
         "--workload", workload, "--steps", "1", "--warmup", "0"],
        capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference-gpu"
    if workload != "ragged":
        assert line["unavailable"]
    else:
        import torch
        if not torch.cuda.is_available():
            assert line["unavailable"]
