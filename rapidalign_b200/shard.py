"""Multi-GPU execution.

Ragged batches: graphs are independent, so each rank computes a share of the
pairs with no collective in the data path; one all_gather returns the
per-graph results to every rank afterwards.

One very large pair (split_pair_kde_mmd_loss): every rank holds the same two
clouds and evaluates every world-th work item (64-row tiles of the x-y, x-x
and y-y blocks, column-split); one all_reduce of the fp64 item partials and
one of the fp32 per-point sums complete the sums on every rank, which then
forms K, the loss and (locally, O(N)) the full gradients.

The partition is a greedy longest-processing-time assignment of the graph
costs N_i^2 + M_i^2 + N_i M_i (the kernel-term count) to the least-loaded
rank; it is deterministic, so every rank computes the same partition locally.
"""
from __future__ import annotations

import heapq
from typing import Callable, List, Optional, Sequence

import numpy as np
import torch

__all__ = ["lpt_partition", "graph_costs", "sharded_pair_results", "split_pair_kde_mmd_loss"]


def graph_costs(nx: Sequence[int], ny: Sequence[int]) -> np.ndarray:
    nx = np.asarray(nx, dtype=np.float64)
    ny = np.asarray(ny, dtype=np.float64)
    return nx * nx + ny * ny + nx * ny


def lpt_partition(cost: Sequence[float], world: int) -> List[np.ndarray]:
    """Indices of the graphs assigned to each of `world` ranks (sorted)."""
    if world < 1:
        raise ValueError("world must be >= 1")
    cost = np.asarray(cost, dtype=np.float64)
    order = np.lexsort((np.arange(cost.size), -cost))  # descending cost, stable by index
    heap = [(0.0, r) for r in range(world)]
    heapq.heapify(heap)
    parts: List[list] = [[] for _ in range(world)]
    for g in order:
        load, r = heapq.heappop(heap)
        parts[r].append(int(g))
        heapq.heappush(heap, (load + float(cost[g]), r))
    return [np.sort(np.array(p, dtype=np.int64)) for p in parts]


def sharded_pair_results(num_graphs: int, costs: Sequence[float],
                         compute: Callable[[np.ndarray], torch.Tensor],
                         group: Optional["torch.distributed.ProcessGroup"] = None) -> torch.Tensor:
    """Run `compute` on this rank's graphs and gather per-graph rows.

    compute(graph_ids) returns a (len(graph_ids), C) tensor of per-graph
    results (e.g. loss, Kxx, Kyy, Kxy) on the rank's device; the return value
    is the (num_graphs, C) tensor in global graph order on every rank.  The
    only collective is one all_gather of zero-padded result blocks.
    """
    import torch.distributed as dist
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    parts = lpt_partition(costs, world)
    mine = parts[rank]
    local = compute(mine)
    C = local.shape[1]
    cap = max(len(p) for p in parts)
    buf = torch.zeros(cap, C, dtype=local.dtype, device=local.device)
    buf[:local.shape[0]] = local
    gathered = [torch.zeros_like(buf) for _ in range(world)]
    dist.all_gather(gathered, buf, group=group)
    out = torch.zeros(num_graphs, C, dtype=local.dtype, device=local.device)
    for r, p in enumerate(parts):
        if len(p):
            out[torch.as_tensor(p, device=local.device)] = gathered[r][:len(p)]
    return out


def split_pair_kde_mmd_loss(x: torch.Tensor, y: torch.Tensor, x_w=None, y_w=None,
                            sigma: float = 0.2, center: bool = True, cosine: bool = False,
                            eps: float = 1e-8, group=None):
    """kde_mmd_loss (rapidalign/kde.py:39-109) for one pair split across the
    ranks of `group` (one process per GPU, NCCL).  Inputs must be identical on
    all ranks; every rank returns the full (loss, Kxx, Kyy, Kxy) and, through
    autograd, the full gradients."""
    import torch.distributed as dist
    from . import _lib
    from ._core import Spec, kde_sums
    from .kde import _loss_from_k, _sigma_value
    if x.ndim != 2 or y.ndim != 2 or x.size(-1) != y.size(-1):
        raise ValueError("x and y must be (N,d) and (M,d) with same d")
    if (isinstance(sigma, torch.Tensor) and bool((sigma <= 0).any())) or \
            (not isinstance(sigma, torch.Tensor) and not sigma > 0):
        raise ValueError("sigma must be positive")
    device = _lib.require_cuda(x, y, x_w, y_w)
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    sig, sig_t = _sigma_value(sigma, device)
    spec = Spec(
        layout=_lib.RA_LAYOUT_DENSE, num_pairs=1, dim=x.shape[1], num_x=x.shape[0],
        num_y=y.shape[0], nmax_x=x.shape[0], nmax_y=y.shape[0],
        weights_x=_lib.RA_WEIGHTS_SUM if x_w is not None else _lib.RA_WEIGHTS_UNIFORM,
        weights_y=_lib.RA_WEIGHTS_SUM if y_w is not None else _lib.RA_WEIGHTS_UNIFORM,
        center=center, sigma=sig, check_errors=(x_w is not None or y_w is not None),
        weight_error_message="weights must sum to a positive value",
        shard_index=rank, shard_count=world)

    def reduce(f64, f32):
        dist.all_reduce(f64, group=group)
        if f32 is not None:
            dist.all_reduce(f32, group=group)

    Kxx, Kyy, Kxy = kde_sums(x, y, x_w, y_w, sig_t, spec,
                             reduce=reduce if world > 1 else None)
    loss = _loss_from_k(Kxx, Kyy, Kxy, cosine, eps)
    dtype = x.dtype
    return loss[0].to(dtype), Kxx[0].to(dtype), Kyy[0].to(dtype), Kxy[0].to(dtype)
