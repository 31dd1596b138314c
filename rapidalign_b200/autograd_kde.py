"""Differentiable segmented KDE loss, drop-in for ``rapidalign.autograd_kde``.

``segmented_kde_loss(x, y, w_x, w_y, ptr_x, ptr_y, sigma)`` returns the
per-pair loss ``Kxx + Kyy - 2 Kxy`` (float64, shape (P,)) with RAW weights and
no centering, exactly as rapidalign/autograd_kde.py:16-129; gradients flow to
x, y, w_x, w_y and the 0-d tensor sigma.  The reference computes its CUDA
forward and backward in two separate passes (three kernels each,
csrc/kde_similarity.cu:283-381 and :607-712, D <= 3 only); here one fused
sm_100a pass produces the sums and the per-point state, and the backward is a
single epilogue launch, for any D.
"""
from __future__ import annotations

import torch

from . import _lib
from ._core import Spec, backward_sums, forward_sums

__all__ = ["segmented_kde_loss", "SegmentedKDELossFunction"]


class SegmentedKDELossFunction(torch.autograd.Function):
    """Same call signature and semantics as rapidalign/autograd_kde.py:16-117."""

    @staticmethod
    def forward(ctx, x, y, w_x, w_y, ptr_x, ptr_y, sigma):
        if sigma.dim() != 0:
            raise ValueError("sigma must be a scalar tensor")
        if ptr_x.numel() != ptr_y.numel():
            raise RuntimeError("ptr_x and ptr_y must have the same length")
        if x.dim() != 2 or y.dim() != 2 or x.size(1) != y.size(1):
            raise RuntimeError("x and y must have shape (N, D) and (M, D)")
        if ptr_x.numel() < 1:
            raise RuntimeError("ptr tensors must contain at least one element")
        if w_x.numel() != x.size(0) or w_y.numel() != y.size(0):
            raise RuntimeError("weights must have one entry per point")
        device = _lib.require_cuda(x, y, w_x, w_y, ptr_x, ptr_y)
        sig = float(sigma.detach().item())
        if not sig > 0:
            raise RuntimeError("sigma must be positive")
        P = ptr_x.numel() - 1
        ctx.state = None
        if P == 0:
            return torch.zeros(0, dtype=torch.float64, device=device)
        spec = Spec(
            layout=_lib.RA_LAYOUT_RAGGED, num_pairs=P, dim=x.shape[1], num_x=x.shape[0],
            num_y=y.shape[0], weights_x=_lib.RA_WEIGHTS_RAW, weights_y=_lib.RA_WEIGHTS_RAW,
            center=False, sigma=sig,
            ptr_x=ptr_x.to(device=device, dtype=torch.long).contiguous(),
            ptr_y=ptr_y.to(device=device, dtype=torch.long).contiguous(),
            check_errors=True)
        need = any(ctx.needs_input_grad[i] for i in (0, 1, 2, 3, 6))
        sigma_t = sigma if ctx.needs_input_grad[6] else None
        K, state = forward_sums(x, y, w_x.reshape(-1), w_y.reshape(-1), sigma_t, spec, need)
        ctx.state = state
        ctx.w_shapes = (w_x.shape, w_y.shape)
        return K[:P] + K[P:2 * P] - 2.0 * K[2 * P:]

    @staticmethod
    def backward(ctx, grad_loss):
        if ctx.state is None:
            return None, None, None, None, None, None, None
        g = grad_loss.to(torch.float64)
        coef = torch.cat([g, g, -2.0 * g])
        n = ctx.needs_input_grad
        gx, gy, gwx, gwy, gs = backward_sums(ctx.state, coef, (n[0], n[1], n[2], n[3], n[6]))
        if gwx is not None:
            gwx = gwx.reshape(ctx.w_shapes[0])
        if gwy is not None:
            gwy = gwy.reshape(ctx.w_shapes[1])
        return gx, gy, gwx, gwy, None, None, gs


def segmented_kde_loss(x, y, w_x, w_y, ptr_x, ptr_y, sigma):
    return SegmentedKDELossFunction.apply(x, y, w_x, w_y, ptr_x, ptr_y, sigma)
