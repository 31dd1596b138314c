"""Multi-GPU sharding of ragged batches: graphs are independent, so each rank
computes a share of the pairs with no collective in the data path; one
all_gather returns the per-graph results to every rank afterwards.

The partition is a greedy longest-processing-time assignment of the graph
costs N_i^2 + M_i^2 + N_i M_i (the kernel-term count) to the least-loaded
rank; it is deterministic, so every rank computes the same partition locally.
"""
from __future__ import annotations

import heapq
from typing import Callable, List, Optional, Sequence

import numpy as np
import torch

__all__ = ["lpt_partition", "graph_costs", "sharded_pair_results"]


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
