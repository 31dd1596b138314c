"""Pairwise-distance spectrum loss on the GPU (rapidalign/algorithms.py).

``pairwise_distance_loss`` keeps the reference's arguments, grouping,
padding, reductions and errors (algorithms.py:19-90): per graph, the sorted
distances of all point pairs of the source and of the target, the shorter
list padded with zeros at its end, the mean squared difference; then
``reduction`` over the graphs.  The per-graph Python loop of the reference
becomes one launch sequence over all graphs (``ra_pdl_forward``: a pair
distance kernel, a segmented sort per graph, a loss kernel per graph) and
the gradient flows back through the sort to the points (``ra_pdl_backward``).
Distances are computed in float32, the sums in float64.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _lib

Tensor = torch.Tensor

__all__ = ["pairwise_distance_loss"]


class _Cloud:
    """One side grouped by batch id: device perm / ptr / pair offsets and the
    host counts the launch sizes need."""

    def __init__(self, points: Tensor, batch: Optional[Tensor]):
        dev = points.device
        if batch is None:
            if points.ndim != 2:
                raise ValueError("points must have shape (N, d)")
            counts = torch.tensor([points.shape[0]], dtype=torch.long, device=dev)
            self.perm = None
        else:
            if points.ndim != 2 or batch.ndim != 1:
                raise ValueError("points must be (N, d) and batch must be (N,)")
            if points.shape[0] != batch.shape[0]:
                raise ValueError("points and batch must have the same length")
            # groups = sorted unique ids; the points of an id keep their order
            _, inverse, counts = torch.unique(batch.to(dev), sorted=True, return_inverse=True,
                                              return_counts=True)
            self.perm = torch.argsort(inverse, stable=True).contiguous()
        zero = torch.zeros(1, dtype=torch.long, device=dev)
        self.ptr = torch.cat([zero, torch.cumsum(counts, 0)]).contiguous()
        pairs = counts * (counts - 1) // 2
        self.poff = torch.cat([zero, torch.cumsum(pairs, 0)]).contiguous()
        stats = torch.stack([pairs.sum(), counts.max() if counts.numel() else zero[0]]).tolist()
        self.groups = counts.numel()
        self.num_pairs, self.max_group = int(stats[0]), int(stats[1])
        self.points = points.detach().to(torch.float32).contiguous()

    def c(self) -> _lib.RaPdlCloud:
        c = _lib.RaPdlCloud()
        c.points = self.points.data_ptr()
        c.perm = _lib.ptr(self.perm)
        c.ptr = self.ptr.data_ptr()
        c.pair_offsets = self.poff.data_ptr()
        c.num_pairs = self.num_pairs
        c.max_group = self.max_group
        return c


class _PairwiseLoss(torch.autograd.Function):
    """(src, tgt) -> per-graph losses (float64 [G])."""

    @staticmethod
    def forward(ctx, src: Tensor, tgt: Tensor, cs: _Cloud, ct: _Cloud):
        lib = _lib.load()
        dev = src.device
        G, D = cs.groups, src.shape[1]
        if cs.max_group > 65536 or ct.max_group > 65536:
            raise ValueError("pairwise_distance_loss: at most 65536 points per graph")
        if cs.num_pairs >= 2 ** 31 or ct.num_pairs >= 2 ** 31:
            raise ValueError("pairwise_distance_loss: at most 2^31 - 1 point pairs per call")
        ws = _lib.workspace(lib.ra_pdl_workspace_bytes(G, cs.num_pairs, ct.num_pairs), dev)
        loss = torch.empty(G, dtype=torch.float64, device=dev)
        a, b = cs.c(), ct.c()
        rc = lib.ra_pdl_forward(ctypes.byref(a), ctypes.byref(b), G, D, loss.data_ptr(),
                                ws.data_ptr(), ws.numel(), _lib.stream_handle(dev))
        _lib.check(rc, "pairwise distance loss")
        ctx.state = (cs, ct, ws, src.dtype, tgt.dtype)
        return loss

    @staticmethod
    def backward(ctx, g_loss: Tensor):
        cs, ct, ws, sdt, tdt = ctx.state
        lib = _lib.load()
        dev = g_loss.device
        G, D = cs.groups, cs.points.shape[1]
        need_s, need_t = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
        gs = torch.zeros_like(cs.points) if need_s else None
        gt = torch.zeros_like(ct.points) if need_t else None
        up = g_loss.to(torch.float64).contiguous()
        a, b = cs.c(), ct.c()
        rc = lib.ra_pdl_backward(ctypes.byref(a), ctypes.byref(b), G, D, up.data_ptr(),
                                 _lib.ptr(gs), _lib.ptr(gt), ws.data_ptr(), ws.numel(),
                                 _lib.stream_handle(dev))
        _lib.check(rc, "pairwise distance loss backward")
        return (gs.to(sdt) if gs is not None else None,
                gt.to(tdt) if gt is not None else None, None, None)


def pairwise_distance_loss(src: Tensor, tgt: Tensor, src_batch: Optional[Tensor] = None,
                           tgt_batch: Optional[Tensor] = None,
                           reduction: str = "mean") -> Tensor:
    """algorithms.py:54-90: loss comparing pairwise distance spectra, invariant
    to rigid transforms, for variable point counts per graph."""
    _lib.require_cuda(src, tgt)
    cs = _Cloud(src, src_batch)
    ct = _Cloud(tgt, tgt_batch)
    if cs.groups != ct.groups:
        raise ValueError("src and tgt batch counts must match")
    if src.shape[1] != tgt.shape[1]:
        raise ValueError("point dimensionality must match per graph")
    if reduction not in ("mean", "sum", "none"):
        raise ValueError(f"Unsupported reduction: {reduction}")
    losses = _PairwiseLoss.apply(src, tgt, cs, ct).to(src.dtype)
    if reduction == "mean":
        return losses.mean()
    if reduction == "sum":
        return losses.sum()
    return losses
