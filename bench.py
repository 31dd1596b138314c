"""Benchmark of the KDE/MMD hot path: Gaussian kernel-term evaluations per
second, forward + backward, through the public API (``pyg_kde_mmd_loss``).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference|reference-gpu]
    torchrun --nproc-per-node N bench.py --gpus N ...        (N > 1)

Workload (a "step"): one forward + backward of ``pyg_kde_mmd_loss`` over a
ragged batch of 4096 graphs, sizes uniform in [32, 2048] points, target
sizes = source size +- uniform [0, 64], coordinates N(0, 1) in 3-D,
target = source + N(0, s^2) noise with s ~ U[0.05, 0.08] per graph,
sigma = 0.25, centering on, sorted batch vectors.  Synthetic, seeded: each
graph is generated from its own seed, so every rank can build its own share
of the batch without generating the rest.

Multi-GPU (default): strong scaling.  The same 4096-graph batch at every N;
graphs are assigned to ranks by a greedy longest-processing-time partition of
their cost N_i^2 + M_i^2 + N_i M_i (rapidalign_b200.shard); ranks compute their
shares with no collective in the data path and the per-graph results are
gathered once after the timed region.  ``--scaling weak`` gives every GPU a
batch of its own size instead (N times the graphs).

Metric: full kernel terms (N^2 + M^2 + N M per graph, the reference's count)
per second over the whole job.  The roofline fraction uses the unique terms
(N(N+1)/2 + M(M+1)/2 + N M) at 16 FP32-pipe operations each, against the FP32
rate measured on the same GPU by a packed-FMA probe kernel.
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

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GRAPHS_PER_GPU = 4096
SIGMA = 0.25
SEED = 20261201
# per unique term: 3 sub + 3 (mul, fma, fma) for r^2, then w = b k, s += w,
# G += w d (5) for the row and the same 5 for the column
FP32_OPS_PER_UNIQUE_TERM = 16
# what the tile kernel issues: nonnegative column weights folded into the
# exponent drop the row-side multiply (15), equal row weights also the
# column-side one (14)
L2_FLUSH_BYTES = 512 << 20     # > 126 MB L2


# ----------------------------------------------------------------------------
# seeded synthetic workloads
# ----------------------------------------------------------------------------

def ragged_graph(g: int, seed: int = SEED, lo: int = 32, hi: int = 2048, dmax: int = 64,
                 dim: int = 3):
    """Graph g of the ragged workload: (src (n, dim), tgt (m, dim)) float32."""
    rng = np.random.default_rng([seed, g])
    n = int(rng.integers(lo, hi + 1))
    m = max(1, n + int(rng.integers(-dmax, dmax + 1)))
    noise = float(rng.uniform(0.05, 0.08))
    src = rng.standard_normal((n, dim)).astype(np.float32)
    base = src[:min(n, m)]
    if m > n:
        base = np.concatenate([base, rng.standard_normal((m - n, dim)).astype(np.float32)])
    tgt = (base + noise * rng.standard_normal((m, dim))).astype(np.float32)
    return src, tgt


def ragged_sizes(graph_ids, seed: int = SEED, lo: int = 32, hi: int = 2048, dmax: int = 64):
    """(n, m) of the given graphs without generating coordinates."""
    out = []
    for g in graph_ids:
        rng = np.random.default_rng([seed, g])
        n = int(rng.integers(lo, hi + 1))
        m = max(1, n + int(rng.integers(-dmax, dmax + 1)))
        out.append((n, m))
    return np.array(out, dtype=np.int64).reshape(-1, 2)


def ragged_batch(graph_ids, seed: int = SEED, **kw):
    """Concatenated batch: x, y (float32), batch_x, batch_y (int64), sizes."""
    xs, ys = [], []
    for g in graph_ids:
        s, t = ragged_graph(int(g), seed, **kw)
        xs.append(s)
        ys.append(t)
    nx = np.array([a.shape[0] for a in xs], dtype=np.int64)
    ny = np.array([a.shape[0] for a in ys], dtype=np.int64)
    x = np.concatenate(xs)
    y = np.concatenate(ys)
    bx = np.repeat(np.arange(len(xs), dtype=np.int64), nx)
    by = np.repeat(np.arange(len(ys), dtype=np.int64), ny)
    return x, y, bx, by, nx, ny


def huge_pair_data(n: int = 262144):
    """The huge-pair workload's clouds: src ~ N(0, 1), tgt = R (src + 0.05
    noise) with R uniform in SO(3)."""
    rng = np.random.default_rng([SEED, 4])
    src = rng.standard_normal((n, 3)).astype(np.float32)
    R = random_rotation(rng)
    tgt = ((src + 0.05 * rng.standard_normal((n, 3))) @ R.T).astype(np.float32)
    return src, tgt


def dense_data(rank: int, B: int = 64, nmax: int = 1024):
    """The dense workload's padded batch of one rank: x, y (B, nmax, 3) and the
    valid lengths lx, ly (prefix masks)."""
    rng = np.random.default_rng([SEED, 2, rank])
    x = rng.standard_normal((B, nmax, 3)).astype(np.float32)
    y = (x + 0.05 * rng.standard_normal((B, nmax, 3))).astype(np.float32)
    lx = rng.integers(512, nmax + 1, B)
    ly = rng.integers(512, nmax + 1, B)
    return x, y, lx, ly


def embed_graph(g: int):
    """Graph g of the embedding workload: n in [64, 512] nodes, D = 128,
    x ~ N(0, 1/D), tgt = src + 0.1 noise."""
    r = np.random.default_rng([SEED, 5, int(g)])
    n = int(r.integers(64, 513))
    a = (r.standard_normal((n, 128)) / np.sqrt(128)).astype(np.float32)
    return a, (a + 0.1 * r.standard_normal((n, 128))).astype(np.float32)


def term_counts(nx: np.ndarray, ny: np.ndarray):
    nx = nx.astype(np.float64)
    ny = ny.astype(np.float64)
    full = float(np.sum(nx * nx + ny * ny + nx * ny))
    unique = float(np.sum(nx * (nx + 1) / 2 + ny * (ny + 1) / 2 + nx * ny))
    return full, unique


# ----------------------------------------------------------------------------
# clocks sampled during the timed region
# ----------------------------------------------------------------------------

class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-i", str(self.gpu), "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, FileNotFoundError):
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()
        # nvidia-smi's start-up (NVML initialisation) can hold the driver for
        # a moment: let it pass before anything is timed
        t0 = time.monotonic()
        while not self.lines and time.monotonic() - t0 < 10.0 and self.proc.poll() is None:
            time.sleep(0.02)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=2)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [v.strip() for v in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx),
                "samples": len(sm), "reasons": sorted(reasons)}


# ----------------------------------------------------------------------------
# CPU baseline: the oracle (C, float64, OpenMP) on a bounded sample
# ----------------------------------------------------------------------------

CPU_BASELINE_WHAT = (
    "the oracle's C port (oracle/kde_oracle.c) of the reference's float64 sums "
    "(rapidalign/kde_gradients.py:39-132): every kernel term of Kxx, Kyy, Kxy and the per-point "
    "sums the gradients are made of, on all host threads; the O(N) centering and "
    "normalisation chain rule is not timed.  The reference's own CPU path is PyTorch "
    "(rapidalign/kde.py), which materialises N x M matrices and needs the reference "
    "package, which is not installed where this bench runs; it ran at ~3e7 terms/s on 8 cores "
    "when measured here, about 40x slower than this port")

def cpu_units(name: str):
    """Units of oracle work (C, float64, OpenMP) drawn from the named workload:
    yields (run, label) where run(cores) computes the forward+backward sums of
    one unit and returns the full kernel terms it covered.  Data generation
    stays outside run()."""
    from oracle import oracle as O
    O.build()
    f64 = lambda v: np.ascontiguousarray(v, dtype=np.float64)
    if name == "huge-pair":
        src, tgt = huge_pair_data()
        x, y = f64(src), f64(tgt)
        n, m = x.shape[0], y.shape[0]
        a, b = np.full(n, 1.0 / n), np.full(m, 1.0 / m)
        rows = 256
        for u in range(10 ** 9):
            side = u % 2
            r0 = (u // 2) * rows % (n if side == 0 else m)
            sel = np.arange(r0, r0 + rows, dtype=np.int64)

            def run(cores, side=side, sel=sel):
                O.rows_sums(side, x, y, a, b, 0.2, sel, nthreads=cores)
                return float(sel.size * (n + m))
            yield run, f"row blocks of {rows} rows of the {n}-point pair (both clouds, cycling)"
    elif name == "dense":
        xb, yb, lx, ly = dense_data(0)
        for c in range(10 ** 9):
            k = c % xb.shape[0]
            x, y = f64(xb[k, :lx[k]]), f64(yb[k, :ly[k]])

            def run(cores, x=x, y=y):
                n, m = x.shape[0], y.shape[0]
                O.raw_sums(x, y, np.full(n, 1.0 / n), np.full(m, 1.0 / m), [0, n], [0, m],
                           SIGMA, nthreads=cores)
                return float(n * n + m * m + n * m)
            yield run, "clouds of the dense batch (valid prefixes, in order, cycling)"
    else:
        for u in range(10 ** 9):
            if name == "embed128":
                sx, sy = embed_graph(u % 1024)
                sigma = 1.0
            else:
                sx, sy = ragged_graph(u % GRAPHS_PER_GPU)
                sigma = SIGMA
            x, y = f64(sx), f64(sy)

            def run(cores, x=x, y=y, sigma=sigma):
                n, m = x.shape[0], y.shape[0]
                O.raw_sums(x, y, np.full(n, 1.0 / n), np.full(m, 1.0 / m), [0, n], [0, m],
                           sigma, nthreads=cores)
                return float(n * n + m * m + n * m)
            yield run, f"graphs of the {name} batch (in order, cycling)"


def cpu_baseline(name: str, budget_s: float = 15.0):
    """The oracle timed on the first units of the same workload until the
    budget is used; full terms/s on every host thread."""
    cores = os.cpu_count() or 1
    total_full, total_t, used, label = 0.0, 0.0, 0, ""
    for run, label in cpu_units(name):
        t0 = time.perf_counter()
        total_full += run(cores)
        total_t += time.perf_counter() - t0
        used += 1
        if total_t > budget_s:
            break
    return {"value": total_full / total_t, "unit": "terms/s", "cores": cores, "kind": "port",
            "sample": f"first {used} {label}, {total_t:.1f} s",
            "what": CPU_BASELINE_WHAT}


# ----------------------------------------------------------------------------
# workloads (one "step" = one forward + backward through the public API)
# ----------------------------------------------------------------------------

def random_rotation(rng) -> np.ndarray:
    """Uniform rotation in SO(3) from a normalised Gaussian quaternion."""
    q = rng.standard_normal(4)
    q /= np.linalg.norm(q)
    w, x, y, z = q
    return np.array([[1 - 2 * (y * y + z * z), 2 * (x * y - z * w), 2 * (x * z + y * w)],
                     [2 * (x * y + z * w), 1 - 2 * (x * x + z * z), 2 * (y * z - x * w)],
                     [2 * (x * z - y * w), 2 * (y * z + x * w), 1 - 2 * (x * x + y * y)]])


def job_graphs(per_batch: int, world: int, scaling: str) -> int:
    """Graphs of the whole job: the batch itself (strong scaling) or one
    batch per GPU (weak scaling)."""
    return per_batch * (world if scaling == "weak" else 1)


class RaggedWorkload:
    """The 4096-graph batch, LPT-partitioned across ranks (strong scaling), or
    4096 graphs per GPU (weak scaling)."""
    issued_ops = 13  # equal weights on both clouds, no weight gradient

    def __init__(self, rank, world, dev, scaling="strong", dim=3, lo=32, hi=2048, sigma=SIGMA,
                 center=True):
        import torch
        from rapidalign_b200.shard import lpt_partition
        self.scaling = scaling
        total = job_graphs(GRAPHS_PER_GPU, world, scaling)
        sizes = ragged_sizes(range(total), lo=lo, hi=hi)
        cost = sizes[:, 0] ** 2 + sizes[:, 1] ** 2 + sizes[:, 0] * sizes[:, 1]
        self.mine = np.sort(lpt_partition(cost, world)[rank])
        x, y, bx, by, nx, ny = ragged_batch(self.mine, lo=lo, hi=hi, dim=dim)
        self.full_local, self.unique_local = term_counts(nx, ny)
        self.sigma, self.center, self.dim = sigma, center, dim
        self.dev = dev
        self.d = {k: torch.from_numpy(v).to(dev) for k, v in
                  dict(x=x, y=y, bx=bx, by=by).items()}
        self.h = {k: torch.from_numpy(v).pin_memory() for k, v in
                  dict(x=x, y=y, bx=bx, by=by).items()}
        self.result_host = torch.empty(len(self.mine), dtype=torch.float32).pin_memory()
        self.config = self.describe(world, scaling)

    @staticmethod
    def describe(world, scaling="strong"):
        total = job_graphs(GRAPHS_PER_GPU, world, scaling)
        sizes = ragged_sizes(range(total))
        full, unique = term_counts(sizes[:, 0], sizes[:, 1])
        return {"workload": f"ragged PyG batch of {GRAPHS_PER_GPU} graphs"
                            f"{' per GPU' if scaling == 'weak' else ''}, 32-2048 points each, "
                            f"D=3, sigma={SIGMA}, centred, pyg_kde_mmd_loss fwd+bwd",
                "graphs": total, "full_terms_per_step": full, "unique_terms_per_step": unique,
                "seed": SEED}

    def step(self, t):
        from rapidalign_b200 import pyg_kde_mmd_loss
        xs = t["x"].detach().requires_grad_(True)
        ys = t["y"].detach().requires_grad_(True)
        loss, _, _, _ = pyg_kde_mmd_loss(xs, ys, src_batch=t["bx"], tgt_batch=t["by"],
                                         sigma=self.sigma, center=self.center)
        loss.sum().backward()
        return loss

    def tiles_time(self, reps):
        from rapidalign_b200 import profiling
        return profiling.tiles_time(self.d["x"], self.d["y"], self.d["bx"], self.d["by"],
                                    self.sigma, reps=reps, center=self.center)


class HugePairWorkload:
    """One pair of N = M = 262144 points split across the ranks (strong
    scaling): src ~ N(0, 1), tgt = R (src + 0.05 noise) with R uniform in
    SO(3), sigma 0.2, centred."""
    issued_ops = 13

    def __init__(self, rank, world, dev, scaling="strong", n=262144, sigma=0.2):
        self.scaling = "strong"  # one pair: the work is fixed whatever N is
        import torch
        import torch.distributed as dist
        src, tgt = huge_pair_data(n)
        self.group = dist.group.WORLD if world > 1 else None
        self.world = world
        full, unique = term_counts(np.array([n]), np.array([n]))
        self.full_local, self.unique_local = full / world, unique / world
        self.full_job, self.unique_job = full, unique
        self.sigma = sigma
        self.dev = dev
        self.d = {"x": torch.from_numpy(src).to(dev), "y": torch.from_numpy(tgt).to(dev)}
        self.h = {"x": torch.from_numpy(src).pin_memory(), "y": torch.from_numpy(tgt).pin_memory()}
        self.result_host = torch.empty(1, dtype=torch.float32).pin_memory()
        self.config = self.describe(world)

    @staticmethod
    def describe(world, scaling="strong"):
        full, unique = term_counts(np.array([262144]), np.array([262144]))
        return {"workload": "single pair N = M = 262144, D=3, tgt = R(src + 0.05 noise), "
                            "sigma=0.2, centred, split over the GPUs by row tiles "
                            "(shard.split_pair_kde_mmd_loss) fwd+bwd",
                "points": 262144, "full_terms_per_step": full, "unique_terms_per_step": unique,
                "seed": SEED}

    def step(self, t):
        from rapidalign_b200.shard import split_pair_kde_mmd_loss
        from rapidalign_b200 import kde_mmd_loss
        xs = t["x"].detach().requires_grad_(True)
        ys = t["y"].detach().requires_grad_(True)
        if self.world > 1:
            loss, _, _, _ = split_pair_kde_mmd_loss(xs, ys, sigma=self.sigma, center=True,
                                                    group=self.group)
        else:
            loss, _, _, _ = kde_mmd_loss(xs, ys, sigma=self.sigma, center=True)
        loss.backward()
        return loss.reshape(1)

    def tiles_time(self, reps):
        from rapidalign_b200 import profiling
        import torch.distributed as dist
        rank = dist.get_rank() if self.world > 1 else 0
        return profiling.tiles_time_pair(self.d["x"], self.d["y"], self.sigma, reps=reps,
                                         shard_index=rank, shard_count=self.world)


class DenseWorkload:
    """Padded batch: B = 64 clouds of Nmax = 1024 points, valid lengths
    uniform in [512, 1024] (prefix masks), tgt = src + 0.05 noise, sigma 0.25,
    centred, kde_mmd_loss_dense fwd+bwd.  Strong scaling: the 64 clouds are
    LPT-partitioned across the ranks; weak: 64 clouds per GPU."""
    issued_ops = 14  # masked (zero) weights: folded, not all equal; no weight gradient

    def __init__(self, rank, world, dev, scaling="strong", B=64, nmax=1024, sigma=SIGMA):
        import torch
        from rapidalign_b200.shard import graph_costs, lpt_partition
        self.scaling = scaling
        if scaling == "weak":
            x, y, lx, ly = dense_data(rank, B, nmax)
        else:
            x, y, lx, ly = dense_data(0, B, nmax)
            mine = np.sort(lpt_partition(graph_costs(lx, ly), world)[rank])
            x, y, lx, ly = x[mine], y[mine], lx[mine], ly[mine]
        mx = np.arange(nmax)[None, :] < lx[:, None]
        my = np.arange(nmax)[None, :] < ly[:, None]
        self.full_local, self.unique_local = term_counts(lx, ly)
        self.sigma = sigma
        self.dev = dev
        self.d = {k: torch.from_numpy(v).to(dev) for k, v in dict(x=x, y=y, mx=mx, my=my).items()}
        self.h = {k: torch.from_numpy(v).pin_memory() for k, v in
                  dict(x=x, y=y, mx=mx, my=my).items()}
        self.result_host = torch.empty(max(len(lx), 1), dtype=torch.float32).pin_memory()
        self.config = self.describe(world, scaling)

    @staticmethod
    def describe(world, scaling="strong"):
        ranks = range(world) if scaling == "weak" else range(1)
        full = unique = 0.0
        for r in ranks:
            _, _, lx, ly = dense_data(r)
            f, u = term_counts(lx, ly)
            full, unique = full + f, unique + u
        return {"workload": "dense padded batch, B=64 clouds of Nmax=1024"
                            f"{' per GPU' if scaling == 'weak' else ''}, valid 512-1024 (prefix "
                            "masks), D=3, sigma=0.25, centred, kde_mmd_loss_dense fwd+bwd",
                "clouds": 64 * len(ranks), "full_terms_per_step": full,
                "unique_terms_per_step": unique, "seed": SEED}

    def step(self, t):
        from rapidalign_b200 import kde_mmd_loss_dense
        xs = t["x"].detach().requires_grad_(True)
        ys = t["y"].detach().requires_grad_(True)
        loss, _, _, _ = kde_mmd_loss_dense(xs, ys, t["mx"], t["my"], sigma=self.sigma,
                                           center=True)
        loss.sum().backward()
        return loss

    def tiles_time(self, reps):
        from rapidalign_b200 import profiling
        return profiling.tiles_time_dense(self.d["x"], self.d["y"], self.d["mx"], self.d["my"],
                                          self.sigma, reps=reps, center=True)


def embed_sizes(total: int) -> np.ndarray:
    return np.array([int(np.random.default_rng([SEED, 5, g]).integers(64, 513))
                     for g in range(total)])


class EmbedWorkload(RaggedWorkload):
    """High-dimensional embeddings: 1024 graphs of 64-512 nodes (per GPU with
    weak scaling), D=128, x ~ N(0, 1/D), tgt = src + 0.1 noise (same sizes),
    sigma 1.0, uncentred."""

    def __init__(self, rank, world, dev, scaling="strong"):
        import torch
        from rapidalign_b200.shard import lpt_partition
        self.scaling = scaling
        total = job_graphs(1024, world, scaling)
        sizes = embed_sizes(total)
        cost = 3.0 * sizes.astype(np.float64) ** 2
        self.mine = np.sort(lpt_partition(cost, world)[rank])
        xs, ys = [], []
        for g in self.mine:
            a, b = embed_graph(int(g))
            xs.append(a)
            ys.append(b)
        nx = np.array([a.shape[0] for a in xs])
        x, y = np.concatenate(xs), np.concatenate(ys)
        bx = np.repeat(np.arange(len(xs)), nx)
        self.full_local, self.unique_local = term_counts(nx, nx)
        # tensor work of one launch of the tensor-core kernel: per graph 4 row-only
        # orientations of ceil(n/128) row tiles x ceil(n/64) column tiles, each a
        # 128 x 64 x 128 Gram GEMM and a 128 x 128 x 64 weighted-sum GEMM,
        # three fp16 products apiece (hi*hi + hi*lo + lo*hi)
        tiles = float(np.sum(4 * np.ceil(nx / 128.0) * np.ceil(nx / 64.0)))
        self.tensor_flops_issued = tiles * 2 * 3 * (2.0 * 128 * 64 * 128)
        self.sigma, self.center, self.dim = 1.0, False, 128
        self.dev = dev
        self.d = {k: torch.from_numpy(v).to(dev) for k, v in
                  dict(x=x, y=y, bx=bx, by=bx).items()}
        self.h = {k: torch.from_numpy(v).pin_memory() for k, v in
                  dict(x=x, y=y, bx=bx, by=bx).items()}
        self.result_host = torch.empty(len(self.mine), dtype=torch.float32).pin_memory()
        self.config = self.describe(world, scaling)

    @staticmethod
    def describe(world, scaling="strong"):
        total = job_graphs(1024, world, scaling)
        n = embed_sizes(total)
        full, unique = term_counts(n, n)
        return {"workload": "graph embeddings, 1024 graphs"
                            f"{' per GPU' if scaling == 'weak' else ''} of 64-512 nodes, D=128, "
                            "sigma=1.0, uncentred, pyg_kde_mmd_loss fwd+bwd",
                "graphs": total, "full_terms_per_step": full, "unique_terms_per_step": unique,
                "seed": SEED}

    def roofline(self, t_tiles, peak_fp32):
        """Tensor roofline: algorithmic flops = full terms x (Gram + weighted
        sum) x 2 D, against the dense fp16 tensor peak (the kernel issues
        kind::f16 MMAs, which run at the measured dense bf16 rate)."""
        peaks = read_measured_peaks()
        measured = bool(peaks and peaks.get("bf16_tflops"))
        bf16 = peaks["bf16_tflops"] if measured else 1590.0  # fallback: earlier pool measurement
        f16 = bf16 * 1e12
        algo = self.full_local * 2 * 2.0 * self.dim
        return {
            "bound": "tensor",
            "achieved": algo / t_tiles / 1e12,
            "peak": f16 / 1e12,
            "unit": "TFLOP/s",
            "frac": algo / t_tiles / f16,
            "peak_source": ("MEASURED_PEAKS.json bf16_tflops" if measured else
                            "fallback 1.59 PFLOP/s bf16") + " (dense fp16 = dense bf16 rate)",
            "kernel": "tilestc16_kernel<128,1> (tcgen05 kind::f16, three fp16 products per GEMM)",
            "kernel_ms": t_tiles * 1e3,
            "flops_per_full_term": 4.0 * self.dim,
            "issued_frac": self.tensor_flops_issued / t_tiles / f16,
            "issued_note": "tensor flops the kernel issues (three fp16 products for fp32 accuracy, "
                           "four row-only orientations, tile padding) over the same peak",
            "traffic": None,
        }


def read_measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return json.load(f)
    except (OSError, ValueError):
        return None


WORKLOADS = {"ragged": RaggedWorkload, "huge-pair": HugePairWorkload, "dense": DenseWorkload,
             "embed128": EmbedWorkload}


# ----------------------------------------------------------------------------
# our arm
# ----------------------------------------------------------------------------

def run_ours(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)

    from rapidalign_b200 import _lib, build as ra_build
    ra_build.build()

    wl = WORKLOADS[args.workload](rank, world, dev, scaling=args.scaling)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    h2d_times = []

    def timed_loop(k, e2e):
        if e2e:
            return e2e_loop(k)
        evs = []
        for _ in range(k):
            flush.fill_(1)  # evict L2 between timed steps (outside the events)
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            wl.step(wl.d)
            e1.record(stream)
            evs.append((e0, e1))
        torch.cuda.synchronize(dev)
        return sum(a.elapsed_time(b) for a, b in evs) / 1e3  # seconds

    from rapidalign_b200.prefetch import DevicePrefetcher
    pf = DevicePrefetcher(dev)  # one copy stream for every e2e loop (warm-up included)
    read_stream = torch.cuda.Stream(dev)

    def e2e_loop(k):
        """k steps fed from pinned host memory through the public API, the
        next step's host-to-device copy staged on a side stream while the
        current step computes (rapidalign_b200.prefetch); each step reads its
        result back to the host.  Timed continuously from before the first
        copy to the end of the last step (the inputs, > L2, are new each step)."""
        torch.cuda.synchronize(dev)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        pf.copy_stream.wait_event(e0)
        pf.put(wl.h)
        copies = []
        for i in range(k):
            t = pf.get()
            copies.append((pf.copy_start, pf.copy_end))
            if i + 1 < k:
                pf.put(wl.h)
            res = wl.step(t)
            # the result goes to the host on a side stream, so the next step's
            # kernels do not queue behind a read waiting for the copy engines
            done = torch.cuda.Event()
            done.record(stream)
            read_stream.wait_event(done)
            with torch.cuda.stream(read_stream):
                wl.result_host.copy_(res.detach().reshape(-1), non_blocking=True)
            res.record_stream(read_stream)
        stream.wait_stream(read_stream)  # the last result is in the timed region
        e1.record(stream)
        torch.cuda.synchronize(dev)
        h2d_times.extend(a.elapsed_time(b) for a, b in copies)
        return e0.elapsed_time(e1) / 1e3  # seconds

    for _ in range(args.warmup):
        wl.step(wl.d)
    if args.profile_step:
        # one more step and exit: the command profiled by ncu (see profiles/)
        wl.step(wl.d)
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.destroy_process_group()
        return
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    launches0 = _lib.launch_count()
    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
    t_dev = timed_loop(args.steps, e2e=False)
    launches = _lib.launch_count() - launches0
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    # one warm-up loop of several steps: it reaches the steady pipeline depth
    # (a batch copying while one computes), so the caching allocator holds the
    # second set of input buffers before the timed loop (1-step loops never
    # stage two batches, and the first timed steps then allocated them)
    timed_loop(max(2, args.warmup), e2e=True)
    t_e2e = timed_loop(args.steps, e2e=True)
    clocks = sampler.stop() if sampler else None

    # the dominant (tile) kernel alone, for the roofline; FP32 peak of this GPU
    t_tiles = wl.tiles_time(max(3, args.steps // 2))
    peak_ops = fp32_peak(dev)

    h2d_local = int(sum(v.numel() * v.element_size() for v in wl.h.values()))
    d2h_local = int(wl.result_host.numel() * 4)
    mine = [t_dev, t_e2e, t_tiles, wl.full_local, wl.unique_local, h2d_local, d2h_local]
    if world > 1:
        per_rank = [torch.zeros(len(mine), dtype=torch.float64, device=dev) for _ in range(world)]
        dist.all_gather(per_rank, torch.tensor(mine, dtype=torch.float64, device=dev))
        per_rank = [t.tolist() for t in per_rank]
    else:
        per_rank = [mine]
    t_dev = max(r[0] for r in per_rank)  # the job's time is the slowest rank's
    t_e2e = max(r[1] for r in per_rank)
    full_all = sum(r[3] for r in per_rank)
    unique_all = sum(r[4] for r in per_rank)
    h2d_all = int(sum(r[5] for r in per_rank))
    d2h_all = int(sum(r[6] for r in per_rank))

    if rank == 0:
        K = args.steps
        value = full_all * K / t_dev
        e2e_value = full_all * K / t_e2e
        roofline = None
        if t_tiles and hasattr(wl, "roofline"):
            roofline = wl.roofline(t_tiles, peak_ops)
        elif t_tiles:
            achieved_ops = wl.unique_local * FP32_OPS_PER_UNIQUE_TERM / t_tiles
            roofline = {
                "bound": "fp32",
                "achieved": achieved_ops / 1e12,
                "peak": peak_ops / 1e12,
                "unit": "Tops/s (FP32-pipe lane ops, FMA = 1)",
                "frac": achieved_ops / peak_ops,
                "peak_source": "measured live: packed-FMA probe kernel (ra_probe_fp32_peak)",
                "kernel": "tiles3_kernel<3> (fused fwd+bwd tile kernel; rank 0)",
                "kernel_ms": t_tiles * 1e3,
                "ops_per_unique_term": FP32_OPS_PER_UNIQUE_TERM,
                "issued_ops_per_unique_term": wl.issued_ops,
                "issued_frac": wl.unique_local * wl.issued_ops / t_tiles / peak_ops,
                "issued_note": "FP32 ops the kernel issues per unique term (weights folded into "
                               "the exponent, no column weight sums without a weight gradient) "
                               "over the same peak",
                "traffic": read_traffic() if args.workload == "ragged" else None,
                "traffic_source": ("dram__bytes_read.sum + dram__bytes_write.sum of one launch, "
                                   "from the committed ncu capture profiles/traffic.json (not "
                                   "measured in this run)") if args.workload == "ragged" else None,
            }
        config = dict(wl.config)
        if abs(config.get("full_terms_per_step", full_all) - full_all) > 1e-6 * full_all:
            raise SystemExit("the ranks' shares do not add up to the configured workload")
        line = {
            "metric": "Gaussian kernel-term evals/sec fwd+bwd",
            "value": value,
            "unit": "terms/s",
            "n_gpus": world,
            "steps": K,
            "warmup": args.warmup,
            "ms_per_step": t_dev / K * 1e3,
            "higher_is_better": True,
            "scaling": wl.scaling,
            "vs_baseline": None,
            "dtype": "f32 (fp64 sums)",
            "data": "synthetic",
            "config": config,
            "method": {
                "l2": "flushed between steps (512 MB write, outside the timed events)",
                "sharding": ("none" if world == 1 else
                             ("work items of the one pair split round-robin, one all-reduce"
                              if args.workload == "huge-pair" else
                              "LPT partition of the graphs across ranks, no collective in "
                              "the step")),
                "time": "CUDA events on the launching stream, max over ranks",
            },
            "per_rank": {
                "ms_per_step": [r[0] / K * 1e3 for r in per_rank],
                "e2e_ms_per_step": [r[1] / K * 1e3 for r in per_rank],
                "tile_kernel_ms": [r[2] * 1e3 for r in per_rank],
                "tile_kernel_ms_min": min(r[2] for r in per_rank) * 1e3,
                "tile_kernel_ms_max": max(r[2] for r in per_rank) * 1e3,
                "full_terms": [r[3] for r in per_rank],
            },
            "e2e": {"value": e2e_value, "unit": "terms/s",
                    "ms_per_step": t_e2e / K * 1e3,
                    "h2d_ms_per_step": (statistics.median(h2d_times[-K:]) if h2d_times else None),
                    "h2d_bytes_per_step": h2d_all,
                    "d2h_bytes_per_step": d2h_all,
                    "pipeline": "each step's inputs copied from pinned host memory on a side "
                                "stream while the previous step computes "
                                "(rapidalign_b200.prefetch.DevicePrefetcher); result read "
                                "back every step; timed continuously over the steps"},
            "gpu_launches": int(launches),
            "roofline": roofline,
            "clocks": clocks,
        }
        if not args.no_cpu_baseline and world == 1:
            line["cpu_baseline"] = cpu_baseline(args.workload, budget_s=args.cpu_budget)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def fp32_peak(dev) -> float:
    import ctypes
    import torch
    from rapidalign_b200 import _lib
    lib = _lib.load()
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    scratch = torch.empty(sms * 8 * 256, dtype=torch.float32, device=dev)
    out = ctypes.c_double(0.0)
    best = 0.0
    for _ in range(3):
        rc = lib.ra_probe_fp32_peak(scratch.data_ptr(), scratch.numel(), 2048, ctypes.byref(out),
                                    _lib.stream_handle(dev))
        _lib.check(rc, "fp32 probe")
        best = max(best, out.value)
    return best


def read_traffic():
    """DRAM bytes per launch of the tile kernel from the committed ncu summary."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    if not os.path.exists(path):
        return None
    try:
        with open(path) as f:
            return json.load(f).get("tiles3_kernel_bytes_per_launch")
    except (OSError, ValueError):
        return None


# ----------------------------------------------------------------------------
# reference arm: the reference's CPU path (here: the oracle port)
# ----------------------------------------------------------------------------

# oracle units per reference step (about a second of host work each)
REFERENCE_UNITS_PER_STEP = {"ragged": 6, "embed128": 8, "dense": 4, "huge-pair": 4}


def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cores = os.cpu_count() or 1
    # each step: a bounded sample of the same workload (the next units)
    per_step = REFERENCE_UNITS_PER_STEP[args.workload]
    units = cpu_units(args.workload)
    times, full, label = [], 0.0, ""
    for s in range(args.warmup + args.steps):
        t_step, f_step = 0.0, 0.0
        for _ in range(per_step):
            run, label = next(units)
            t0 = time.perf_counter()
            f_step += run(cores)
            t_step += time.perf_counter() - t0
        if s >= args.warmup:
            times.append(t_step)
            full += f_step
    value = full / sum(times)
    wl = WORKLOADS[args.workload]
    config = dict(wl.describe(world, args.scaling))
    line = {
        "impl": "reference",
        "metric": "Gaussian kernel-term evals/sec fwd+bwd",
        "value": value,
        "unit": "terms/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": sum(times) / len(times) * 1e3,
        "higher_is_better": True,
        "scaling": "strong" if args.workload == "huge-pair" else args.scaling,
        "vs_baseline": None,
        "dtype": "f64",
        "data": "synthetic",
        "config": config,
        "cpu_baseline": {"value": value, "unit": "terms/s", "cores": cores, "kind": "port",
                         "sample": f"{per_step} {label} per step", "what": CPU_BASELINE_WHAT},
        "e2e": {"value": value, "unit": "terms/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------
# the reference's own GPU kernels (context: the same box, the same batch)
# ----------------------------------------------------------------------------

REF_GPU_UNAVAILABLE = {
    "embed128": "the reference's segmented backward holds a point's difference in a "
                "3-element array (csrc/kde_similarity.cu), so it is undefined for D > 3",
    "dense": "the reference's dense op is forward-only (no dense backward in its extension)",
    "huge-pair": "the reference puts one pair on one thread block: a 262144-point pair "
                 "would take hours",
}


def run_reference_gpu(args):
    """The reference's CUDA extension (its csrc/ sources built for sm_100a by
    baseline/build_ref_cuda.py) on the same 4096-graph batch, as its
    segmented_kde_loss runs it: kde_mmd_forward_segmented, the loss
    Kxx + Kyy - 2 Kxy, then kde_mmd_backward_segmented with dL/dloss = 1.
    Raw weights 1/n per graph, points as given (that path has no centring);
    the kernel terms per step are the same as ours."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    base = {"impl": "reference-gpu", "metric": "Gaussian kernel-term evals/sec fwd+bwd",
            "unit": "terms/s", "higher_is_better": True}
    if args.workload in REF_GPU_UNAVAILABLE:
        print(json.dumps(dict(base, unavailable=REF_GPU_UNAVAILABLE[args.workload])), flush=True)
        return
    import glob
    import importlib.util
    import torch
    hits = sorted(glob.glob(os.path.join(ROOT, "baseline", "_ref", "rapidalign_ref_cuda*.so")))
    if not hits or not torch.cuda.is_available():
        why = "the reference extension is not built (baseline/build_ref_cuda.py)" if not hits \
            else "no CUDA device"
        print(json.dumps(dict(base, unavailable=why)), flush=True)
        return
    spec = importlib.util.spec_from_file_location("rapidalign_ref_cuda", hits[0])
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    wl = RaggedWorkload(0, 1, dev)
    x, y = wl.d["x"].contiguous(), wl.d["y"].contiguous()
    P = len(wl.mine)
    cnt_x = torch.bincount(wl.d["bx"], minlength=P)
    cnt_y = torch.bincount(wl.d["by"], minlength=P)
    zero = torch.zeros(1, dtype=torch.long, device=dev)
    px = torch.cat([zero, torch.cumsum(cnt_x, 0)])
    py = torch.cat([zero, torch.cumsum(cnt_y, 0)])
    wx = (1.0 / cnt_x.clamp_min(1).double()).repeat_interleave(cnt_x).float()
    wy = (1.0 / cnt_y.clamp_min(1).double()).repeat_interleave(cnt_y).float()
    g = torch.ones(P, dtype=torch.float64, device=dev)
    sigma = float(wl.sigma)
    stream = torch.cuda.current_stream(dev)
    flush = torch.empty(512 << 20, dtype=torch.uint8, device=dev)

    def step():
        kxx, kyy, kxy = ref.kde_mmd_forward_segmented(x, y, wx, wy, px, py, sigma)
        loss = kxx + kyy - 2.0 * kxy
        ref.kde_mmd_backward_segmented(x, y, wx, wy, px, py, g, sigma)
        return loss

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    evs = []
    loss = None
    for _ in range(args.steps):
        flush.fill_(1)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        loss = step()
        e1.record(stream)
        evs.append((e0, e1))
    torch.cuda.synchronize(dev)
    t = sum(a.elapsed_time(b) for a, b in evs) / 1e3
    config = dict(wl.describe(1, "strong"))
    line = dict(base, value=wl.full_local * args.steps / t, n_gpus=1, steps=args.steps,
                warmup=args.warmup, ms_per_step=t / args.steps * 1e3, scaling="strong",
                vs_baseline=None, dtype="f64 (fp32 inputs)", data="synthetic", config=config,
                what="the reference's segmented CUDA forward + backward (one thread block per "
                     "pair, fp64), weights 1/n per graph, no centring",
                loss_mean=float(loss.mean()))
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference", "reference-gpu"],
                    help="ours; reference (its CPU path: the fp64 port on the host cores); "
                         "reference-gpu (its own CUDA kernels, built by baseline/build_ref_cuda.py)")
    ap.add_argument("--workload", default="ragged", choices=sorted(WORKLOADS),
                    help="ragged (default, the headline workload), huge-pair, dense, embed128")
    ap.add_argument("--scaling", default="strong", choices=["strong", "weak"],
                    help="strong (default): the same batch at every GPU count; weak: one batch "
                         "per GPU")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-budget", type=float, default=15.0)
    ap.add_argument("--profile-step", action="store_true",
                    help="warm-up steps plus one step, no timing or output (for ncu)")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.impl == "reference-gpu":
        run_reference_gpu(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
