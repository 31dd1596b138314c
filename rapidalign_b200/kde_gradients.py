"""Float64 closed-form KDE/MMD forward and backward on the GPU
(rapidalign/kde_gradients.py).

The reference keeps these helpers as a trusted float64 verification path
(``kde_mmd_forward_cpu``, ``kde_mmd_backward_cpu``,
``kde_mmd_backward_ragged_cpu``, kde_gradients.py:39-193).  Here the same
functions run on CUDA tensors through the library's float64 kernels
(``ra_kde_exact_f64`` for the sums and gradients, ``ra_kde_exact_matrices_f64``
for the dense kernel and difference matrices), with the reference's argument
meaning, return types and errors.  They evaluate every term in double
precision in a direct O(N^2 D) loop: meant for small problems and for
checking the fast fused path, like their originals.

Loss per pair: L = Kxx + Kyy - 2 Kxy with raw weights (no normalisation, no
centering); the gradients are those of L.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict

import torch

from . import _lib

Tensor = torch.Tensor


@dataclass
class KDEForwardResult:
    loss: Tensor
    Kxx: Tensor
    Kyy: Tensor
    Kxy: Tensor
    Gxx: Tensor
    Gyy: Tensor
    Gxy: Tensor
    diff_xx: Tensor
    diff_yy: Tensor
    diff_xy: Tensor


_PTR_ERRORS = {
    _lib.RA_ERR_PTR_START: "ptr must start at 0",
    _lib.RA_ERR_PTR_END: "ptr[-1] must equal number of nodes",
    _lib.RA_ERR_PTR_ORDER: "ptr offsets must match node stacks",
}


def _matrices(a: Tensor, b: Tensor, sigma: float):
    """kde_gradients.py:32-36: (G [n, m], diff [n, m, D]) in float64."""
    lib = _lib.load()
    n, m, D = a.shape[0], b.shape[0], a.shape[1]
    G = torch.empty((n, m), dtype=torch.float64, device=a.device)
    diff = torch.empty((n, m, D), dtype=torch.float64, device=a.device)
    rc = lib.ra_kde_exact_matrices_f64(_lib.ptr(a), n, _lib.ptr(b), m, D, float(sigma),
                                       _lib.ptr(G), _lib.ptr(diff), _lib.stream_handle(a.device))
    _lib.check(rc, "kde exact matrices")
    return G, diff


def _exact(x: Tensor, y: Tensor, w_x: Tensor, w_y: Tensor, ptr_x: Tensor, ptr_y: Tensor,
           sigma: float, grads: bool):
    """Per-pair loss, K sums and (optionally) all gradients, float64."""
    lib = _lib.load()
    dev = x.device
    P = ptr_x.numel() - 1
    NX, NY, D = x.shape[0], y.shape[0], x.shape[1]
    x, y = x.contiguous(), y.contiguous()
    w_x, w_y = w_x.contiguous().reshape(-1), w_y.contiguous().reshape(-1)
    ptr_x = ptr_x.to(device=dev, dtype=torch.long).contiguous()
    ptr_y = ptr_y.to(device=dev, dtype=torch.long).contiguous()
    f64 = dict(dtype=torch.float64, device=dev)
    out = {k: torch.empty(P, **f64) for k in ("loss", "Kxx", "Kyy", "Kxy")}
    if grads:
        out.update(x=torch.empty((NX, D), **f64), y=torch.empty((NY, D), **f64),
                   w_x=torch.empty(NX, **f64), w_y=torch.empty(NY, **f64),
                   sigma_per_pair=torch.empty(P, **f64))
    ws = _lib.workspace(lib.ra_kde_exact_workspace_bytes(NX, NY), dev)
    g = (lambda k: _lib.ptr(out[k]) if grads else None)
    rc = lib.ra_kde_exact_f64(
        _lib.ptr(x), _lib.ptr(y), _lib.ptr(w_x), _lib.ptr(w_y), _lib.ptr(ptr_x), _lib.ptr(ptr_y),
        P, NX, NY, D, float(sigma), _lib.ptr(out["loss"]), _lib.ptr(out["Kxx"]),
        _lib.ptr(out["Kyy"]), _lib.ptr(out["Kxy"]), g("x"), g("y"), g("w_x"), g("w_y"),
        g("sigma_per_pair"), ws.data_ptr(), ws.numel(), _lib.stream_handle(dev))
    if rc in _PTR_ERRORS:  # the messages of the fused path (kde.py:133-149)
        raise ValueError(_PTR_ERRORS[rc])
    _lib.check(rc, "kde exact")
    return out


def _single(x: Tensor, y: Tensor, w_x: Tensor, w_y: Tensor, sigma: float, grads: bool):
    dev = _lib.require_cuda(x, y, w_x, w_y)
    ptr_x = torch.tensor([0, x.shape[0]], dtype=torch.long, device=dev)
    ptr_y = torch.tensor([0, y.shape[0]], dtype=torch.long, device=dev)
    return _exact(x, y, w_x, w_y, ptr_x, ptr_y, sigma, grads)


def kde_mmd_forward(x: Tensor, y: Tensor, w_x: Tensor, w_y: Tensor,
                    sigma: float) -> KDEForwardResult:
    """kde_gradients.py:39-73: K sums, loss and the dense G / diff matrices
    of one pair (float64 inputs, as the reference requires)."""
    if x.dtype != torch.float64 or y.dtype != torch.float64:
        raise ValueError("kde_mmd_forward_cpu expects float64 tensors for stability")
    out = _single(x, y, w_x, w_y, sigma, grads=False)
    Gxx, diff_xx = _matrices(x, x, sigma)
    Gyy, diff_yy = _matrices(y, y, sigma)
    Gxy, diff_xy = _matrices(x, y, sigma)
    return KDEForwardResult(loss=out["loss"][0], Kxx=out["Kxx"][0], Kyy=out["Kyy"][0],
                            Kxy=out["Kxy"][0], Gxx=Gxx, Gyy=Gyy, Gxy=Gxy, diff_xx=diff_xx,
                            diff_yy=diff_yy, diff_xy=diff_xy)


def kde_mmd_backward(x: Tensor, y: Tensor, w_x: Tensor, w_y: Tensor,
                     sigma: float) -> Dict[str, Tensor]:
    """kde_gradients.py:76-132: analytic gradients of one pair's loss with
    respect to x, y, w_x, w_y and sigma, plus the forward result."""
    if x.dtype != torch.float64 or y.dtype != torch.float64:
        raise ValueError("kde_mmd_backward_cpu expects float64 tensors")
    out = _single(x, y, w_x, w_y, sigma, grads=True)
    fwd = kde_mmd_forward(x, y, w_x, w_y, sigma)
    return {"x": out["x"], "y": out["y"], "w_x": out["w_x"], "w_y": out["w_y"],
            "sigma": out["sigma_per_pair"][0], "forward": fwd}


def kde_mmd_backward_ragged(x: Tensor, y: Tensor, w_x: Tensor, w_y: Tensor, ptr_x: Tensor,
                            ptr_y: Tensor, sigma: float) -> Dict[str, Tensor]:
    """kde_gradients.py:135-193: per-pair losses, K sums and gradients of a
    ragged batch (pairs given by ptr_x / ptr_y) in one launch sequence."""
    if not (x.dtype == y.dtype == w_x.dtype == w_y.dtype == torch.float64):
        raise ValueError("ragged backward expects float64 tensors")
    if ptr_x.numel() != ptr_y.numel():
        raise ValueError("ptr_x and ptr_y must have the same length")
    _lib.require_cuda(x, y, w_x, w_y)
    out = _exact(x, y, w_x, w_y, ptr_x, ptr_y, sigma, grads=True)
    return {"x": out["x"], "y": out["y"], "w_x": out["w_x"], "w_y": out["w_y"],
            "sigma_per_pair": out["sigma_per_pair"],
            "sigma_total": out["sigma_per_pair"].sum(), "loss": out["loss"],
            "Kxx": out["Kxx"], "Kyy": out["Kyy"], "Kxy": out["Kxy"]}


# the reference's names (their float64 semantics are kept; the work runs on
# the tensors' CUDA device)
kde_mmd_forward_cpu = kde_mmd_forward
kde_mmd_backward_cpu = kde_mmd_backward
kde_mmd_backward_ragged_cpu = kde_mmd_backward_ragged

__all__ = [
    "KDEForwardResult",
    "kde_mmd_forward",
    "kde_mmd_backward",
    "kde_mmd_backward_ragged",
    "kde_mmd_forward_cpu",
    "kde_mmd_backward_cpu",
    "kde_mmd_backward_ragged_cpu",
]
