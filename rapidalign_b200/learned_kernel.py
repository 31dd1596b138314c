"""Learned KDE/MMD kernels (rapidalign/learned_kernel.py) on the B200 path.

The same modules with the same parameters (names, shapes and
initialisation, so state dicts load either way): every kernel sum goes
through the fused CUDA kernels (:func:`rapidalign_b200.kde_mmd_loss`, and
:func:`rapidalign_b200.kde_mmd_loss_bands` for the multi-band module: all
bandwidths in one call), with gradients to the positions (and so to the
anisotropic scale), to the node weights (and so to the weight network) and
to sigma.

* ``NodeWeightNet``   -- learned_kernel.py:23-38
* ``LearnedKernel``   -- learned_kernel.py:41-115 (multi-band, gated)
* ``SingleSigmaKernel`` -- learned_kernel.py:118-158
* ``StructuredKernel``  -- learned_kernel.py:161-202

The gate statistics of ``LearnedKernel`` (mean and variance of the pairwise
distances, learned_kernel.py:16-20 and 103-110) are computed as in the
reference, from the full distance matrix in PyTorch, and carry no gradient
(the reference rebuilds them with ``torch.tensor``).
"""
from __future__ import annotations

import math
from typing import Sequence

import torch
import torch.nn.functional as F
from torch import nn

from .kde import kde_mmd_loss, kde_mmd_loss_bands

Tensor = torch.Tensor


def _full_cdist(a: Tensor, b: Tensor) -> Tensor:
    """Pairwise Euclidean distances in the reference's form
    (learned_kernel.py:16-20): sqrt(clamp(|a|^2 + |b|^2 - 2 a.b, 0))."""
    a2 = (a * a).sum(dim=1, keepdim=True)
    b2 = (b * b).sum(dim=1, keepdim=True).T
    return (a2 + b2 - 2.0 * (a @ b.T)).clamp_min(0.0).sqrt()


class NodeWeightNet(nn.Module):
    """Positive, normalised node weights from point coordinates or features."""

    def __init__(self, in_feats: int = 2, hidden: int = 32):
        super().__init__()
        self.mlp = nn.Sequential(nn.Linear(in_feats, hidden), nn.ReLU(), nn.Linear(hidden, 1))

    def forward(self, pos: Tensor) -> Tensor:
        weights = F.softplus(self.mlp(pos)) + 1e-6
        weights = weights / weights.sum()
        return weights.squeeze(-1)


class LearnedKernel(nn.Module):
    """Multi-scale KDE/MMD loss: one MMD per bandwidth, mixed by a gate driven
    by pair statistics, with learnable bandwidths, anisotropic axis scales
    and node weights."""

    def __init__(self, sigmas: Sequence[float] = (0.05, 0.1, 0.2), learn_scale: bool = True,
                 use_weight_net: bool = True, gated: bool = True, coord_dim: int = 2):
        super().__init__()
        self.log_sigmas = nn.Parameter(torch.log(torch.tensor(sigmas, dtype=torch.float32)))
        self.use_weight_net = use_weight_net
        self.learn_scale = learn_scale
        self.coord_dim = coord_dim
        if use_weight_net:
            self.weight_net = NodeWeightNet(in_feats=coord_dim)
        if learn_scale:
            self.log_scale = nn.Parameter(torch.zeros(coord_dim))
        hidden = 32
        self.gate = nn.Sequential(nn.Linear(4, hidden), nn.ReLU(), nn.Linear(hidden, len(sigmas)))
        self.bias = nn.Parameter(torch.zeros(1))

    def _scale_points(self, pts: Tensor) -> Tensor:
        return pts * torch.exp(self.log_scale) if self.learn_scale else pts

    def _weights(self, pts: Tensor) -> Tensor:
        if not self.use_weight_net:
            return torch.full((pts.size(0),), 1.0 / pts.size(0), device=pts.device,
                              dtype=pts.dtype)
        return self.weight_net(pts)

    def forward(self, base_points: Tensor, target_points: Tensor) -> Tensor:
        base = self._scale_points(base_points)
        target = self._scale_points(target_points)
        w_base = self._weights(base)
        w_target = self._weights(target)
        per_band = kde_mmd_loss_bands(base, target, w_base, w_target,
                                      sigmas=torch.exp(self.log_sigmas), center=True)[0]
        with torch.no_grad():
            dist = _full_cdist(base, target)
            stats = torch.stack([
                dist.mean(), dist.var(),
                torch.tensor(abs(float(base.size(0) - target.size(0))) / (base.size(0) + 1e-6),
                             device=base.device, dtype=dist.dtype),
                w_base.var() + w_target.var()]).to(base.dtype)
        weights = F.softplus(self.gate(stats.float()))
        weights = weights / weights.sum()
        return (weights * per_band).sum() + self.bias.squeeze()


class SingleSigmaKernel(nn.Module):
    """Single-band KDE/MMD loss with optional node weights and anisotropy."""

    def __init__(self, init_sigma: float = 0.1, learn_scale: bool = True,
                 use_weight_net: bool = False, coord_dim: int = 2):
        super().__init__()
        self.log_sigma = nn.Parameter(torch.tensor(math.log(init_sigma), dtype=torch.float32))
        self.learn_scale = learn_scale
        self.use_weight_net = use_weight_net
        self.coord_dim = coord_dim
        if learn_scale:
            self.log_scale = nn.Parameter(torch.zeros(coord_dim))
        if use_weight_net:
            self.weight_net = NodeWeightNet(in_feats=coord_dim)

    def _scale_points(self, pts: Tensor) -> Tensor:
        return pts * torch.exp(self.log_scale) if self.learn_scale else pts

    def _weights(self, pts: Tensor) -> Tensor:
        if not self.use_weight_net:
            return torch.full((pts.size(0),), 1.0 / pts.size(0), device=pts.device,
                              dtype=pts.dtype)
        return self.weight_net(pts)

    def forward(self, base_points: Tensor, target_points: Tensor) -> Tensor:
        base = self._scale_points(base_points)
        target = self._scale_points(target_points)
        loss, _, _, _ = kde_mmd_loss(base, target, self._weights(base), self._weights(target),
                                     sigma=torch.exp(self.log_sigma), center=True)
        return loss


class StructuredKernel(nn.Module):
    """Single-band KDE/MMD loss with node weights from structural features and
    a descriptor-driven scale."""

    def __init__(self, init_sigma: float = 0.1, learn_scale: bool = True, feature_dim: int = 5,
                 descriptor_dim: int = 4):
        super().__init__()
        self.log_sigma = nn.Parameter(torch.tensor(math.log(init_sigma), dtype=torch.float32))
        self.learn_scale = learn_scale
        if learn_scale:
            self.log_scale = nn.Parameter(torch.zeros(2))
        self.weight_net = NodeWeightNet(in_feats=feature_dim)
        self.descriptor_gate = nn.Sequential(nn.Linear(descriptor_dim, 32), nn.ReLU(),
                                             nn.Linear(32, 1))
        self.bias = nn.Parameter(torch.zeros(1))

    def _scale_points(self, pts: Tensor) -> Tensor:
        return pts * torch.exp(self.log_scale) if self.learn_scale else pts

    def forward(self, base: dict, target: dict) -> Tensor:
        base_pos = self._scale_points(base["pos"])
        target_pos = self._scale_points(target["pos"])
        loss, _, _, _ = kde_mmd_loss(base_pos, target_pos, self.weight_net(base["feat"]),
                                     self.weight_net(target["feat"]),
                                     sigma=torch.exp(self.log_sigma), center=True)
        desc_diff = torch.abs(base["desc"] - target["desc"])
        scale = F.softplus(self.descriptor_gate(desc_diff)) + 1e-6
        return loss * scale.squeeze() + self.bias.squeeze()


__all__ = ["LearnedKernel", "NodeWeightNet", "SingleSigmaKernel", "StructuredKernel"]
