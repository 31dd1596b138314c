"""Measurement helpers: device time of the hot tile kernel alone, for the
roofline of the ragged forward+backward (CUDA events recorded by the library
on the launch stream around that one launch)."""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._core import Spec, _f32, _inputs
from .kde import _ensure_ptr


def tiles_time(x: torch.Tensor, y: torch.Tensor, batch_x: torch.Tensor, batch_y: torch.Tensor,
               sigma: float, reps: int = 5, center: bool = True, need_grad: bool = True) -> float:
    """Mean seconds of the fused tile kernel for the pyg_kde_mmd_loss problem
    (uniform weights) with gradients requested."""
    lib = _lib.load()
    dev = x.device
    ptr_x, P, _ = _ensure_ptr(None, batch_x, x.shape[0], dev)
    ptr_y, _, _ = _ensure_ptr(None, batch_y, y.shape[0], dev)
    spec = Spec(layout=_lib.RA_LAYOUT_RAGGED, num_pairs=P, dim=x.shape[1], num_x=x.shape[0],
                num_y=y.shape[0], center=center, sigma=sigma, ptr_x=ptr_x, ptr_y=ptr_y,
                skip_weight_sums=True)
    x32, y32 = _f32(x), _f32(y)
    desc = spec.desc(need_grad, False)
    inp = _inputs(x32, y32, None, None, spec)
    ws = _lib.workspace(lib.ra_kde_workspace_bytes(ctypes.byref(desc)), dev)
    K = torch.empty(3 * P, dtype=torch.float64, device=dev)
    ms = ctypes.c_float(0.0)
    total = 0.0
    with torch.cuda.device(dev):
        for r in range(reps + 1):
            rc = lib.ra_kde_forward_profiled(ctypes.byref(desc), ctypes.byref(inp), K.data_ptr(),
                                             ws.data_ptr(), ws.numel(),
                                             _lib.stream_handle(dev), ctypes.byref(ms))
            _lib.check(rc, "profiled forward")
            if r > 0:  # first run warms up
                total += ms.value
    return total / reps / 1e3


def tiles_time_dense(x: torch.Tensor, y: torch.Tensor, mask_x: torch.Tensor,
                     mask_y: torch.Tensor, sigma: float, reps: int = 5,
                     center: bool = True) -> float:
    """Mean seconds of the tile kernel for the kde_mmd_loss_dense problem
    (padded (B, N, D) clouds with masks, no weights) with gradients requested."""
    lib = _lib.load()
    dev = x.device
    B = x.shape[0]
    mx = mask_x.to(device=dev, dtype=torch.uint8).contiguous()
    my = mask_y.to(device=dev, dtype=torch.uint8).contiguous()
    spec = Spec(layout=_lib.RA_LAYOUT_DENSE, num_pairs=B, dim=x.shape[2],
                num_x=B * x.shape[1], num_y=B * y.shape[1], nmax_x=x.shape[1],
                nmax_y=y.shape[1], weights_x=_lib.RA_WEIGHTS_SUM_CLAMPED,
                weights_y=_lib.RA_WEIGHTS_SUM_CLAMPED, center=center, sigma=sigma,
                mask_x=mx, mask_y=my, skip_weight_sums=True)
    x32, y32 = _f32(x), _f32(y)
    desc = spec.desc(True, False)
    inp = _inputs(x32, y32, None, None, spec)
    ws = _lib.workspace(lib.ra_kde_workspace_bytes(ctypes.byref(desc)), dev)
    K = torch.empty(3 * B, dtype=torch.float64, device=dev)
    ms = ctypes.c_float(0.0)
    total = 0.0
    with torch.cuda.device(dev):
        for r in range(reps + 1):
            rc = lib.ra_kde_forward_profiled(ctypes.byref(desc), ctypes.byref(inp), K.data_ptr(),
                                             ws.data_ptr(), ws.numel(),
                                             _lib.stream_handle(dev), ctypes.byref(ms))
            _lib.check(rc, "profiled forward")
            if r > 0:  # first run warms up
                total += ms.value
    return total / reps / 1e3


def tiles_time_pair(x: torch.Tensor, y: torch.Tensor, sigma: float, reps: int = 3,
                    center: bool = True, shard_index: int = 0, shard_count: int = 1) -> float:
    """Mean seconds of the tile kernel for one pair (kde_mmd_loss with uniform
    weights and gradients), or of this shard's items of a split evaluation."""
    lib = _lib.load()
    dev = x.device
    spec = Spec(layout=_lib.RA_LAYOUT_DENSE, num_pairs=1, dim=x.shape[1], num_x=x.shape[0],
                num_y=y.shape[0], nmax_x=x.shape[0], nmax_y=y.shape[0], center=center,
                sigma=sigma, shard_index=shard_index, shard_count=shard_count,
                skip_weight_sums=True)
    x32, y32 = _f32(x), _f32(y)
    desc = spec.desc(True, False)
    inp = _inputs(x32, y32, None, None, spec)
    ws = _lib.workspace(lib.ra_kde_workspace_bytes(ctypes.byref(desc)), dev)
    K = torch.empty(3, dtype=torch.float64, device=dev)
    ms = ctypes.c_float(0.0)
    total = 0.0
    with torch.cuda.device(dev):
        for r in range(reps + 1):
            rc = lib.ra_kde_forward_profiled(ctypes.byref(desc), ctypes.byref(inp), K.data_ptr(),
                                             ws.data_ptr(), ws.numel(),
                                             _lib.stream_handle(dev), ctypes.byref(ms))
            _lib.check(rc, "profiled forward")
            if r > 0:
                total += ms.value
    return total / reps / 1e3
