"""Generate ``tests/golden/oracle/huge_pair_262144.npz``: the fp64 oracle's values for
the single-pair workload of 262144 points per cloud.

    python tests/golden/oracle/make_huge_pair_fixture.py      (a few minutes on 8 cores)

The reference cannot evaluate this pair at all: its PyTorch path materialises
N x M matrices (rapidalign/kde.py:83-101, 275 GB here) and its CUDA kernels
put one pair on one thread block (csrc/kde_similarity.cu:196-233).  So the
reference values come from the oracle (``oracle/kde_oracle.c``, a float64 restatement of
rapidalign/kde_gradients.py:39-132, with the centering and chain rules of
``oracle/oracle.py``), run once over the whole pair here and stored:

* Kxx, Kyy, Kxy and the loss (MMD, centred, uniform weights, sigma 0.2) --
  every term of the pair, 2.06e11 of them, in float64;
* the gradients of the loss w.r.t. x and y on a seeded subset of 256 rows of
  each cloud (the rows' exact float64 values; a full gradient would make the
  fixture megabytes).

The inputs are ``bench.huge_pair_data()`` (seeded), regenerated identically
by the test, so only results are stored.  This folder holds fixtures made by
the oracle; the folder above holds those made by running the reference.
"""
from __future__ import annotations

import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(os.path.dirname(HERE)))
sys.path.insert(0, ROOT)

N_POINTS = 262144
SIGMA = 0.2
SUBSET = 256
SUBSET_SEED = 424242
OUT = os.path.join(HERE, "huge_pair_262144.npz")


def subset_rows(n: int) -> np.ndarray:
    rng = np.random.default_rng(SUBSET_SEED)
    return np.sort(rng.choice(n, SUBSET, replace=False)).astype(np.int64)


def main() -> None:
    import bench
    from oracle import oracle as O
    src, tgt = bench.huge_pair_data(N_POINTS)
    t0 = time.time()
    r = O.kde_mmd_loss(src, tgt, sigma=SIGMA, center=True, upstream=[1.0, 0.0, 0.0, 0.0])
    dt = time.time() - t0
    rows = subset_rows(N_POINTS)
    np.savez(OUT, n=N_POINTS, sigma=SIGMA, rows=rows, loss=r.loss, Kxx=r.Kxx, Kyy=r.Kyy,
             Kxy=r.Kxy, grad_x_rows=r.grad_x[rows], grad_y_rows=r.grad_y[rows],
             grad_x_absmax=np.max(np.abs(r.grad_x)), grad_y_absmax=np.max(np.abs(r.grad_y)))
    print(f"wrote {OUT} ({dt:.0f} s of oracle work): loss {float(r.loss):.12e} "
          f"Kxx {float(r.Kxx):.12e} Kyy {float(r.Kyy):.12e} Kxy {float(r.Kxy):.12e}")


if __name__ == "__main__":
    main()
