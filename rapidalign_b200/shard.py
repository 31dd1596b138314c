"""Multi-GPU execution.

Ragged batches: graphs are independent, so each rank computes a share of the
pairs with no collective in the data path; one all_gather returns the
per-graph results to every rank afterwards.

One very large pair (split_pair_kde_mmd_loss): every rank holds the same two
clouds and evaluates every world-th work item (64-row tiles of the x-y, x-x
and y-y blocks, column-split); ONE all_reduce of a float64 buffer that packs
the item partials of K and the per-point sums completes the sums on every
rank, which then forms K, the loss and (locally, O(N)) the full gradients.

Batches as a library feature (sharded_pyg_kde_mmd_loss,
sharded_kde_mmd_loss_dense): every rank passes the whole batch, computes the
loss of its LPT share of the graphs (clouds) and gathers every graph's
(loss, Kxx, Kyy, Kxy); gradients flow to the rank's own graphs only (data
parallel: each rank's backward covers its share).

The partition is a greedy longest-processing-time assignment of the graph
costs N_i^2 + M_i^2 + N_i M_i (the kernel-term count) to the least-loaded
rank; it is deterministic, so every rank computes the same partition locally.
"""
from __future__ import annotations

import heapq
from typing import Callable, List, Optional, Sequence

import numpy as np
import torch

__all__ = ["lpt_partition", "graph_costs", "sharded_pair_results", "split_pair_kde_mmd_loss",
           "packed_all_reduce", "sharded_pyg_kde_mmd_loss", "sharded_kde_mmd_loss_dense"]


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


def packed_all_reduce(f64: torch.Tensor, f32: Optional[torch.Tensor], group=None) -> None:
    """Sum a float64 and a float32 buffer over the group in place with ONE
    collective: both are packed into one float64 buffer (the float32 values
    are summed in float64 and rounded once)."""
    import torch.distributed as dist
    if f32 is None:
        dist.all_reduce(f64, group=group)
        return
    n64 = f64.numel()
    buf = torch.empty(n64 + f32.numel(), dtype=torch.float64, device=f64.device)
    buf[:n64].copy_(f64)
    buf[n64:].copy_(f32)
    dist.all_reduce(buf, group=group)
    f64.copy_(buf[:n64])
    f32.copy_(buf[n64:])


def _scatter_rows(local: torch.Tensor, gathered: torch.Tensor, mine: np.ndarray) -> torch.Tensor:
    """The gathered per-graph values with this rank's rows replaced by its own
    (differentiable) results."""
    out = gathered.detach().clone()
    idx = torch.as_tensor(mine, device=local.device, dtype=torch.long)
    return out.index_put((idx,), local)


def _sharded(num: int, costs, compute, group):
    """compute(ids) -> (loss, Kxx, Kyy, Kxy) of the rank's graphs; returns the
    four (num,) tensors of all graphs on every rank."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    mine = lpt_partition(costs, world)[rank]
    holder = {}

    def run(ids):
        outs = compute(ids)
        holder["outs"] = outs
        return torch.stack([o.detach().to(torch.float64) for o in outs], dim=1)

    gathered = sharded_pair_results(num, costs, run, group)
    outs = holder["outs"]
    return tuple(_scatter_rows(o.to(torch.float64), gathered[:, k], mine).to(o.dtype)
                 for k, o in enumerate(outs))


def sharded_pyg_kde_mmd_loss(src_pos: torch.Tensor, tgt_pos: torch.Tensor, src_ptr, tgt_ptr,
                             group=None, **kw):
    """``pyg_kde_mmd_loss`` (rapidalign/kde.py:302-428) of a ragged batch split
    over the ranks of ``group``: each rank passes the whole batch (positions
    and ptr offsets), evaluates its LPT share of the graphs on its GPU and
    returns the (loss, Kxx, Kyy, Kxy) of every graph; its backward gives the
    gradients of its own graphs' points (zeros elsewhere).  One all_gather."""
    from .kde import pyg_kde_mmd_loss
    px = torch.as_tensor(src_ptr).detach().cpu().numpy().astype(np.int64)
    py = torch.as_tensor(tgt_ptr).detach().cpu().numpy().astype(np.int64)
    if px.size != py.size:
        raise ValueError("source and target batches must have the same length")
    nx, ny = np.diff(px), np.diff(py)
    dev = src_pos.device
    sw, tw = kw.pop("src_w", None), kw.pop("tgt_w", None)

    def compute(ids):
        ids = np.asarray(ids, dtype=np.int64)
        xi = np.concatenate([np.arange(px[g], px[g + 1]) for g in ids]) if ids.size else \
            np.zeros(0, np.int64)
        yi = np.concatenate([np.arange(py[g], py[g + 1]) for g in ids]) if ids.size else \
            np.zeros(0, np.int64)
        xt = torch.as_tensor(xi, device=dev)
        yt = torch.as_tensor(yi, device=dev)
        lp_x = torch.as_tensor(np.concatenate([[0], np.cumsum(nx[ids])]), device=dev)
        lp_y = torch.as_tensor(np.concatenate([[0], np.cumsum(ny[ids])]), device=dev)
        return pyg_kde_mmd_loss(src_pos.index_select(0, xt), tgt_pos.index_select(0, yt),
                                src_ptr=lp_x, tgt_ptr=lp_y,
                                src_w=None if sw is None else sw.reshape(-1).index_select(0, xt),
                                tgt_w=None if tw is None else tw.reshape(-1).index_select(0, yt),
                                **kw)

    return _sharded(nx.size, graph_costs(nx, ny), compute, group)


def sharded_kde_mmd_loss_dense(x: torch.Tensor, y: torch.Tensor, mask_x: torch.Tensor,
                               mask_y: torch.Tensor, group=None, x_w=None, y_w=None, **kw):
    """``kde_mmd_loss_dense`` (rapidalign/kde.py:211-299) of a padded batch
    split over the ranks of ``group`` by the LPT partition of the clouds'
    valid-point costs: each rank passes the whole batch, evaluates its share
    of the rows and returns the (B,) results of every row; its backward gives
    the gradients of its own rows.  One all_gather."""
    from .kde import kde_mmd_loss_dense
    cx = mask_x.detach().sum(1).cpu().numpy()
    cy = mask_y.detach().sum(1).cpu().numpy()
    dev = x.device

    def compute(ids):
        idx = torch.as_tensor(np.asarray(ids, dtype=np.int64), device=dev)
        return kde_mmd_loss_dense(x.index_select(0, idx), y.index_select(0, idx),
                                  mask_x.index_select(0, idx), mask_y.index_select(0, idx),
                                  x_w=None if x_w is None else x_w.index_select(0, idx),
                                  y_w=None if y_w is None else y_w.index_select(0, idx), **kw)

    return _sharded(x.shape[0], graph_costs(cx, cy), compute, group)


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
    from ._core import mmd_outputs
    from .kde import _sigma_value
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

    Kxx, Kyy, Kxy = kde_sums(x, y, x_w, y_w, sig_t, spec,
                             reduce=(lambda f64, f32: packed_all_reduce(f64, f32, group))
                             if world > 1 else None)
    loss, Kxx, Kyy, Kxy = mmd_outputs(Kxx, Kyy, Kxy, cosine, eps, x.dtype)
    return loss[0], Kxx[0], Kyy[0], Kxy[0]
