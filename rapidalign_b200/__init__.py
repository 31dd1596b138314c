"""rapidalign_b200 -- B200-native (sm_100a) KDE/MMD loss, API-compatible with
``rapidalign`` (kde_mmd_loss, kde_mmd_loss_dense, pyg_kde_mmd_loss and the
differentiable segmented_kde_loss)."""
from .kde import (batch_ptrs, kde_mmd_loss, kde_mmd_loss_bands, kde_mmd_loss_dense,
                  pyg_batch_kde_mmd_loss, pyg_kde_mmd_loss)
from .algorithms import pairwise_distance_loss
from .autograd_kde import SegmentedKDELossFunction, segmented_kde_loss

__all__ = [
    "kde_mmd_loss",
    "kde_mmd_loss_bands",
    "kde_mmd_loss_dense",
    "pyg_kde_mmd_loss",
    "pyg_batch_kde_mmd_loss",
    "batch_ptrs",
    "segmented_kde_loss",
    "pairwise_distance_loss",
    "SegmentedKDELossFunction",
]
