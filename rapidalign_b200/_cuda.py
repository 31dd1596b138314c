"""Legacy extension op set, drop-in for the ``rapidalign._cuda`` pybind module
(csrc/bindings.cpp:34-71).  Same three names, positional arguments, checks
(RuntimeError, as TORCH_CHECK raises) and output dtypes; each call goes
through one C-ABI entry point of ``librapidalign_b200.so`` on the current
stream, with outputs and workspace allocated by torch.
"""
from __future__ import annotations

import torch

from . import _lib

__all__ = ["kde_mmd_forward", "kde_mmd_forward_segmented", "kde_mmd_backward_segmented"]


def _check(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


def kde_mmd_forward(x, y, w_x, w_y, mask_x, mask_y, sigma: float):
    """Dense masked forward (csrc/kde_similarity.cu:84-192) -> (Kxx, Kyy, Kxy) f64 [B]."""
    _check(x.is_cuda, "kde_mmd_forward_cuda: x must be CUDA tensor")
    _check(y.is_cuda, "kde_mmd_forward_cuda: y must be CUDA tensor")
    _check(x.dtype == torch.float32, "kde_mmd_forward_cuda: x must be float32")
    _check(y.dtype == torch.float32, "kde_mmd_forward_cuda: y must be float32")
    _check(x.dim() == 3 and y.dim() == 3 and x.size(2) == y.size(2),
           "x and y must have shape (B, N, D)")
    _check(sigma > 0.0, "sigma must be positive")
    B, Nx, D = x.shape
    Ny = y.shape[1]
    _check(w_x.dim() == 2 and w_x.size(0) == B and w_x.size(1) == Nx,
           "w_x must have shape (B, Nx)")
    _check(w_y.dim() == 2 and w_y.size(0) == B and w_y.size(1) == Ny,
           "w_y must have shape (B, Ny)")
    _check(w_x.dtype == torch.float32, "kde_mmd_forward_segmented_cuda: w_x must be float32")
    _check(w_y.dtype == torch.float32, "kde_mmd_forward_segmented_cuda: w_y must be float32")
    _check(mask_x.dim() == 2 and mask_x.size(0) == B and mask_x.size(1) == Nx,
           "mask_x must have shape (B, Nx)")
    _check(mask_y.dim() == 2 and mask_y.size(0) == B and mask_y.size(1) == Ny,
           "mask_y must have shape (B, Ny)")
    _check(y.size(0) == B, "x and y must have shape (B, N, D)")
    lib = _lib.load()
    dev = x.device
    x, y = x.contiguous(), y.contiguous()
    wx, wy = w_x.to(dev).contiguous(), w_y.to(dev).contiguous()
    mx = mask_x.to(dev).to(torch.uint8).contiguous()
    my = mask_y.to(dev).to(torch.uint8).contiguous()
    K = torch.zeros(3, B, dtype=torch.float64, device=dev)
    if B == 0:
        return K[0], K[1], K[2]
    ws = _lib.workspace(lib.ra_kde_mmd_forward_workspace_bytes(B, Nx, Ny, D), dev)
    with torch.cuda.device(dev):
        rc = lib.ra_kde_mmd_forward(x.data_ptr(), y.data_ptr(), wx.data_ptr(), wy.data_ptr(),
                                    mx.data_ptr(), my.data_ptr(), B, Nx, Ny, D, float(sigma),
                                    K[0].data_ptr(), K[1].data_ptr(), K[2].data_ptr(),
                                    ws.data_ptr(), ws.numel(), _lib.stream_handle(dev))
    _lib.check(rc, "kde_mmd_forward")
    return K[0], K[1], K[2]


def _seg_checks(name, x, y, w_x, w_y, ptr_x, ptr_y, sigma):
    _check(x.is_cuda, f"{name}: x must be CUDA tensor")
    _check(y.is_cuda, f"{name}: y must be CUDA tensor")
    _check(ptr_x.is_cuda, f"{name}: ptr_x must be CUDA tensor")
    _check(ptr_y.is_cuda, f"{name}: ptr_y must be CUDA tensor")
    _check(x.dtype == torch.float32, f"{name}: x must be float32")
    _check(y.dtype == torch.float32, f"{name}: y must be float32")
    _check(w_x.dtype == torch.float32, f"{name}: w_x must be float32")
    _check(w_y.dtype == torch.float32, f"{name}: w_y must be float32")
    _check(ptr_x.dtype == torch.int64, f"{name}: ptr_x must be int64")
    _check(ptr_y.dtype == torch.int64, f"{name}: ptr_y must be int64")
    _check(x.dim() == 2 and y.dim() == 2 and x.size(1) == y.size(1),
           "x and y must have shape (N, D) and (M, D)")
    _check(ptr_x.dim() == 1 and ptr_y.dim() == 1, "ptr_x and ptr_y must be 1-D")
    _check(ptr_x.numel() >= 1 and ptr_y.numel() >= 1,
           "ptr tensors must contain at least one element")
    _check(ptr_x.numel() == ptr_y.numel(), "ptr_x and ptr_y must have the same length")
    _check(sigma > 0.0, "sigma must be positive")
    _check(w_x.numel() == x.size(0) and w_y.numel() == y.size(0),
           f"{name}: weights must have one entry per point")


def _raise_device_error(lib, ws, dev):
    code = lib.ra_kde_check(ws.data_ptr(), _lib.stream_handle(dev))
    if code != _lib.RA_OK:
        raise RuntimeError(f"rapidalign_b200: {_lib.status_string(code)}")


def kde_mmd_forward_segmented(x, y, w_x, w_y, ptr_x, ptr_y, sigma: float):
    """Ragged forward (csrc/kde_similarity.cu:283-381) -> (Kxx, Kyy, Kxy) f64 [P]."""
    name = "kde_mmd_forward_segmented_cuda"
    _seg_checks(name, x, y, w_x, w_y, ptr_x, ptr_y, sigma)
    lib = _lib.load()
    dev = x.device
    P = ptr_x.numel() - 1
    K = torch.zeros(3, P, dtype=torch.float64, device=dev)
    if P == 0:
        return K[0], K[1], K[2]
    x, y = x.contiguous(), y.contiguous()
    wx, wy = w_x.contiguous(), w_y.contiguous()
    px, py = ptr_x.contiguous(), ptr_y.contiguous()
    NX, NY, D = x.shape[0], y.shape[0], x.shape[1]
    ws = _lib.workspace(lib.ra_kde_mmd_forward_segmented_workspace_bytes(P, NX, NY, D), dev)
    with torch.cuda.device(dev):
        rc = lib.ra_kde_mmd_forward_segmented(
            x.data_ptr(), y.data_ptr(), wx.data_ptr(), wy.data_ptr(), px.data_ptr(),
            py.data_ptr(), P, NX, NY, D, float(sigma), K[0].data_ptr(), K[1].data_ptr(),
            K[2].data_ptr(), ws.data_ptr(), ws.numel(), _lib.stream_handle(dev))
        _lib.check(rc, name)
        _raise_device_error(lib, ws, dev)
    return K[0], K[1], K[2]


def kde_mmd_backward_segmented(x, y, w_x, w_y, ptr_x, ptr_y, grad_loss, sigma: float):
    """Ragged backward (csrc/kde_similarity.cu:607-712) ->
    (grad_x f32, grad_y f32, grad_wx f64, grad_wy f64, grad_sigma_pairs f64 [P])."""
    name = "kde_mmd_backward_segmented_cuda"
    _check(x.is_cuda, f"{name}: x must be CUDA tensor")
    _check(y.is_cuda, f"{name}: y must be CUDA tensor")
    _check(w_x.is_cuda and w_y.is_cuda, "weights must be CUDA tensors")
    _check(ptr_x.is_cuda and ptr_y.is_cuda, "ptr tensors must be CUDA tensors")
    _check(grad_loss.is_cuda, "grad_loss must be CUDA tensor")
    _check(grad_loss.dtype == torch.float64, "grad_loss must be float64")
    _seg_checks(name, x, y, w_x, w_y, ptr_x, ptr_y, sigma)
    lib = _lib.load()
    dev = x.device
    P = ptr_x.numel() - 1
    _check(grad_loss.numel() == P, "grad_loss must have one entry per pair")
    x, y = x.contiguous(), y.contiguous()
    NX, NY, D = x.shape[0], y.shape[0], x.shape[1]
    gx = torch.zeros_like(x)
    gy = torch.zeros_like(y)
    gwx = torch.zeros(NX, dtype=torch.float64, device=dev)
    gwy = torch.zeros(NY, dtype=torch.float64, device=dev)
    gs = torch.zeros(P, dtype=torch.float64, device=dev)
    if P == 0:
        return gx, gy, gwx, gwy, gs
    ws = _lib.workspace(lib.ra_kde_mmd_backward_segmented_workspace_bytes(P, NX, NY, D), dev)
    with torch.cuda.device(dev):
        rc = lib.ra_kde_mmd_backward_segmented(
            x.data_ptr(), y.data_ptr(), w_x.contiguous().data_ptr(),
            w_y.contiguous().data_ptr(), ptr_x.contiguous().data_ptr(),
            ptr_y.contiguous().data_ptr(), P, NX, NY, D, grad_loss.contiguous().data_ptr(),
            float(sigma), gx.data_ptr(), gy.data_ptr(), gwx.data_ptr(), gwy.data_ptr(),
            gs.data_ptr(), ws.data_ptr(), ws.numel(), _lib.stream_handle(dev))
        _lib.check(rc, name)
        _raise_device_error(lib, ws, dev)
    return gx, gy, gwx, gwy, gs
