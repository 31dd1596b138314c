"""Public KDE/MMD loss API, drop-in for ``rapidalign.kde``.

Same names, arguments, return values and error messages as the reference:

* ``kde_mmd_loss``        rapidalign/kde.py:39-109   (single pair)
* ``kde_mmd_loss_dense``  rapidalign/kde.py:211-299  (padded batch + masks)
* ``pyg_kde_mmd_loss``    rapidalign/kde.py:302-428  (ragged PyG-style batch)

each returning ``(loss, Kxx, Kyy, Kxy)``.  The sums are computed by the
sm_100a kernels of ``librapidalign_b200.so`` in one fused pass; unlike the
reference CUDA branch, every output is differentiable (w.r.t. positions,
weights and a tensor ``sigma``) through the centering and weight
normalisation.  The K sums are float64; the results are cast to the input
dtype as the reference does (kde.py:269-274, 372-377).

Inputs must be CUDA tensors: there is no CPU fallback.  Argument checks that
need no device data run first and raise the reference's ``ValueError``s.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from . import _lib
from ._core import GraphCountMismatch, Spec, kde_sums, mmd_outputs

Tensor = torch.Tensor

__all__ = ["kde_mmd_loss", "kde_mmd_loss_bands", "kde_mmd_loss_dense", "pyg_kde_mmd_loss",
           "pyg_batch_kde_mmd_loss", "batch_ptrs"]


def _sigma_value(sigma, device) -> Tuple[float, Optional[Tensor]]:
    """sigma as a float for the kernels, plus the tensor if gradients flow to it."""
    if isinstance(sigma, Tensor):
        if sigma.numel() != 1:
            raise ValueError("sigma must be a scalar")
        val = float(sigma.detach().reshape(()).item())
        return val, (sigma.reshape(()) if sigma.requires_grad else None)
    return float(sigma), None


def kde_mmd_loss(
    x: Tensor,
    y: Tensor,
    x_w: Optional[Tensor] = None,
    y_w: Optional[Tensor] = None,
    sigma: float = 0.2,
    center: bool = True,
    cosine: bool = False,
    eps: float = 1e-8,
) -> Tuple[Tensor, Tensor, Tensor, Tensor]:
    """RKHS distance (MMD^2) or cosine loss between two weighted point sets.

    Args match rapidalign/kde.py:39-63: x (N, d), y (M, d), optional weights
    (normalised to sum 1), Gaussian bandwidth sigma (float or scalar tensor,
    differentiable), weighted-centroid centering, cosine variant.
    Returns 0-d tensors (loss, Kxx, Kyy, Kxy) in x's dtype.
    """
    if x.ndim != 2 or y.ndim != 2 or x.size(-1) != y.size(-1):
        raise ValueError("x and y must be (N,d) and (M,d) with same d")
    if isinstance(sigma, Tensor):
        if (sigma <= 0).any():
            raise ValueError("sigma must be positive")
    elif not sigma > 0:
        raise ValueError("sigma must be positive")
    if x_w is not None and x_w.numel() != x.shape[0]:
        raise ValueError("weights length must equal number of nodes")
    if y_w is not None and y_w.numel() != y.shape[0]:
        raise ValueError("weights length must equal number of nodes")
    # an empty weight vector sums to 0 (kde.py:24-26)
    if (x_w is not None and x_w.numel() == 0) or (y_w is not None and y_w.numel() == 0):
        raise ValueError("weights must sum to a positive value")
    device = _lib.require_cuda(x, y, x_w, y_w)
    dtype = x.dtype
    sig, sig_t = _sigma_value(sigma, device)
    spec = Spec(
        layout=_lib.RA_LAYOUT_DENSE, num_pairs=1, dim=x.shape[1],
        num_x=x.shape[0], num_y=y.shape[0], nmax_x=x.shape[0], nmax_y=y.shape[0],
        weights_x=_lib.RA_WEIGHTS_SUM if x_w is not None else _lib.RA_WEIGHTS_UNIFORM,
        weights_y=_lib.RA_WEIGHTS_SUM if y_w is not None else _lib.RA_WEIGHTS_UNIFORM,
        center=center, sigma=sig,
        check_errors=(x_w is not None or y_w is not None),
        weight_error_message="weights must sum to a positive value")
    Kxx, Kyy, Kxy = kde_sums(x, y, x_w, y_w, sig_t, spec)
    loss, Kxx, Kyy, Kxy = mmd_outputs(Kxx, Kyy, Kxy, cosine, eps, dtype)
    return loss[0], Kxx[0], Kyy[0], Kxy[0]


def kde_mmd_loss_bands(
    x: Tensor,
    y: Tensor,
    x_w: Optional[Tensor] = None,
    y_w: Optional[Tensor] = None,
    sigmas=(0.05, 0.1, 0.2),
    center: bool = True,
    cosine: bool = False,
    eps: float = 1e-8,
) -> Tuple[Tensor, Tensor, Tensor, Tensor]:
    """``kde_mmd_loss`` for S bandwidths of one pair of clouds in one call.

    Equivalent to ``[kde_mmd_loss(x, y, x_w, y_w, sigma=s, ...) for s in
    sigmas]`` stacked (the multi-band use of rapidalign/learned_kernel.py:89-
    115): returns (loss, Kxx, Kyy, Kxy) of shape (S,).  The S bands run as S
    pairs of one launch sequence with a per-pair bandwidth, so a small cloud
    pays the fixed cost of the fused pipeline once instead of S times.
    ``sigmas`` is a sequence of floats or a 1-D tensor (differentiable: each
    band gets its own gradient).
    """
    if x.ndim != 2 or y.ndim != 2 or x.size(-1) != y.size(-1):
        raise ValueError("x and y must be (N,d) and (M,d) with same d")
    if x_w is not None and x_w.numel() != x.shape[0]:
        raise ValueError("weights length must equal number of nodes")
    if y_w is not None and y_w.numel() != y.shape[0]:
        raise ValueError("weights length must equal number of nodes")
    if (x_w is not None and x_w.numel() == 0) or (y_w is not None and y_w.numel() == 0):
        raise ValueError("weights must sum to a positive value")
    device = _lib.require_cuda(x, y, x_w, y_w)
    sig = sigmas if isinstance(sigmas, Tensor) else torch.tensor(list(sigmas),
                                                                 dtype=torch.float64)
    if sig.ndim != 1 or sig.numel() == 0:
        raise ValueError("sigmas must be a non-empty 1-D sequence")
    sig64 = sig.detach().to(device=device, dtype=torch.float64).contiguous()
    if bool((sig64 <= 0).any()):
        raise ValueError("sigma must be positive")
    S, N, M, D = sig.numel(), x.shape[0], y.shape[0], x.shape[1]
    dtype = x.dtype
    spec = Spec(
        layout=_lib.RA_LAYOUT_DENSE, num_pairs=S, dim=D, num_x=S * N, num_y=S * M,
        nmax_x=N, nmax_y=M,
        weights_x=_lib.RA_WEIGHTS_SUM if x_w is not None else _lib.RA_WEIGHTS_UNIFORM,
        weights_y=_lib.RA_WEIGHTS_SUM if y_w is not None else _lib.RA_WEIGHTS_UNIFORM,
        center=center, sigma=1.0, sigma_pairs=sig64,
        check_errors=(x_w is not None or y_w is not None),
        weight_error_message="weights must sum to a positive value")
    # the bands as S rows of a dense batch (gradients of the repeats add up)
    xr = x.unsqueeze(0).expand(S, N, D)
    yr = y.unsqueeze(0).expand(S, M, D)
    xwr = None if x_w is None else x_w.reshape(1, N).expand(S, N)
    ywr = None if y_w is None else y_w.reshape(1, M).expand(S, M)
    sig_t = sig.to(device) if isinstance(sigmas, Tensor) and sigmas.requires_grad else None
    Kxx, Kyy, Kxy = kde_sums(xr, yr, xwr, ywr, sig_t, spec)
    return mmd_outputs(Kxx, Kyy, Kxy, cosine, eps, dtype)


def kde_mmd_loss_dense(
    x: Tensor,
    y: Tensor,
    mask_x: Tensor,
    mask_y: Tensor,
    x_w: Optional[Tensor] = None,
    y_w: Optional[Tensor] = None,
    sigma: float = 0.2,
    center: bool = True,
    cosine: bool = False,
    eps: float = 1e-8,
):
    """Batched KDE/MMD loss on dense padded tensors (rapidalign/kde.py:211-299).

    x, y: (B, Nmax, D); mask_x, mask_y: (B, Nmax) bool (any pattern; a prefix
    mask lets the kernels skip the padded tail entirely); optional weights
    (B, Nmax), default uniform over valid nodes.  Returns (B,) tensors.
    """
    if isinstance(sigma, Tensor):
        if (sigma <= 0).any():
            raise ValueError("sigma must be positive")
    elif sigma <= 0:
        raise ValueError("sigma must be positive")
    if x.ndim != 3 or y.ndim != 3 or x.size(0) != y.size(0) or x.size(2) != y.size(2):
        raise ValueError("x and y must have shape (B, Nmax, D)")
    if mask_x.shape != x.shape[:2] or mask_y.shape != y.shape[:2]:
        raise ValueError("masks must have shape (B, Nmax)")
    if x_w is not None and x_w.shape != x.shape[:2]:
        raise ValueError("weights must have shape (B, Nmax)")
    if y_w is not None and y_w.shape != y.shape[:2]:
        raise ValueError("weights must have shape (B, Nmax)")
    device = _lib.require_cuda(x, y)
    dtype = x.dtype
    B = x.shape[0]
    if B == 0:
        zero = torch.zeros((0,), device=device, dtype=dtype)
        return zero, zero, zero, zero
    sig, sig_t = _sigma_value(sigma, device)
    mx = mask_x.to(device=device, dtype=torch.bool).to(torch.uint8).contiguous()
    my = mask_y.to(device=device, dtype=torch.bool).to(torch.uint8).contiguous()
    spec = Spec(
        layout=_lib.RA_LAYOUT_DENSE, num_pairs=B, dim=x.shape[2],
        num_x=B * x.shape[1], num_y=B * y.shape[1], nmax_x=x.shape[1], nmax_y=y.shape[1],
        weights_x=_lib.RA_WEIGHTS_SUM_CLAMPED, weights_y=_lib.RA_WEIGHTS_SUM_CLAMPED,
        center=center, sigma=sig, mask_x=mx, mask_y=my, check_errors=False)
    xw = None if x_w is None else x_w.to(device)
    yw = None if y_w is None else y_w.to(device)
    Kxx, Kyy, Kxy = kde_sums(x, y, xw, yw, sig_t, spec)
    return mmd_outputs(Kxx, Kyy, Kxy, cosine, eps, dtype)


def _read_back(values: Tensor) -> list:
    """A few device values on the host, waiting only for the current stream
    (a pinned copy plus an event, where ``tolist()`` would wait for the
    device's default stream too)."""
    host = torch.empty(values.shape, dtype=values.dtype, pin_memory=True)
    host.copy_(values, non_blocking=True)
    done = torch.cuda.Event()
    done.record(torch.cuda.current_stream(values.device))
    done.synchronize()
    return host.tolist()


def _ensure_ptr(ptr: Optional[Tensor], batch: Optional[Tensor], total_nodes: int,
                device) -> Tuple[Tensor, int, bool]:
    """kde.py:124-156.  Returns (ptr, num_graphs, user_given).  The value
    checks of a user ptr (first/last entry, order) run on the device inside
    the forward and raise the same ValueErrors."""
    if ptr is not None:
        ptr = ptr.to(device=device, dtype=torch.long).contiguous()
        if ptr.dim() != 1:
            raise ValueError("ptr must be 1-D")
        if ptr.numel() == 0:
            raise ValueError("ptr must have at least one element")
        return ptr, ptr.numel() - 1, True

    if batch is None:
        raise ValueError("either ptr or batch must be provided")

    batch = batch.to(device=device, dtype=torch.long).contiguous()
    if batch.numel() != total_nodes:
        raise ValueError("batch length must match number of nodes")
    if batch.numel() == 0:
        return torch.zeros(1, dtype=torch.long, device=device), 0, False
    # one synchronisation for both the order check and the graph count
    if batch.numel() > 1:
        unsorted = (batch[:-1] > batch[1:]).any()
        info = _read_back(torch.stack([unsorted.to(torch.long), batch[-1], batch[0]]))
    else:
        info = [0, int(batch[0].item()), int(batch[0].item())]
    if info[0]:
        raise ValueError("batch indices must be sorted for contiguous blocks")
    if info[2] < 0:
        raise ValueError("batch indices must be non-negative")
    num_graphs = int(info[1]) + 1
    # sorted batch -> ptr[g] = first index with batch >= g
    bounds = torch.arange(num_graphs + 1, device=device, dtype=torch.long)
    ptr = torch.searchsorted(batch, bounds, right=False).contiguous()
    return ptr, num_graphs, False


def _ensure_ptrs(src_ptr: Optional[Tensor], src_batch: Optional[Tensor], n_src: int,
                 tgt_ptr: Optional[Tensor], tgt_batch: Optional[Tensor], n_tgt: int,
                 device) -> Tuple[Tensor, int, bool, Tensor, int, bool]:
    """_ensure_ptr for both sides with a single host synchronisation when
    both come as batch vectors (the checks and graph counts of the two sides
    are read back together); same results and errors, source side first."""
    if src_ptr is not None or tgt_ptr is not None or src_batch is None or tgt_batch is None:
        return (*_ensure_ptr(src_ptr, src_batch, n_src, device),
                *_ensure_ptr(tgt_ptr, tgt_batch, n_tgt, device))
    sb = src_batch.to(device=device, dtype=torch.long).contiguous()
    tb = tgt_batch.to(device=device, dtype=torch.long).contiguous()
    if sb.numel() != n_src or tb.numel() != n_tgt:
        raise ValueError("batch length must match number of nodes")
    if sb.numel() < 2 or tb.numel() < 2:
        return (*_ensure_ptr(None, sb, n_src, device), *_ensure_ptr(None, tb, n_tgt, device))
    info = _read_back(torch.stack([(sb[:-1] > sb[1:]).any().to(torch.long), sb[-1], sb[0],
                                   (tb[:-1] > tb[1:]).any().to(torch.long), tb[-1], tb[0]]))
    out = []
    for b, (unsorted, last, first) in ((sb, info[:3]), (tb, info[3:])):
        if unsorted:
            raise ValueError("batch indices must be sorted for contiguous blocks")
        if first < 0:
            raise ValueError("batch indices must be non-negative")
        num_graphs = int(last) + 1
        bounds = torch.arange(num_graphs + 1, device=device, dtype=torch.long)
        out += [torch.searchsorted(b, bounds, right=False).contiguous(), num_graphs, False]
    return tuple(out)


def batch_ptrs(src_batch: Tensor, tgt_batch: Tensor) -> Tuple[Tensor, Tensor]:
    """ptr offsets of two sorted batch vectors (kde.py:124-156 semantics and
    errors), with one host synchronisation for both; on the current stream.
    ``pyg_kde_mmd_loss(..., src_ptr=, tgt_ptr=)`` then needs none."""
    ps, _, _, pt, _, _ = _ensure_ptrs(None, src_batch, src_batch.numel(), None, tgt_batch,
                                      tgt_batch.numel(), src_batch.device)
    return ps, pt


# Graph count of the last batch-vector call on each device: a batch-vector
# call starts its work with this count, builds ptr on the device and verifies
# the count there; a wrong guess is found before any result is returned and
# the call is repeated with the exact count.  The first call on a device (and
# a repeat) reads the count back instead.
_GRAPH_COUNT_HINT: dict = {}


def _batch_ptrs_on_device(sb: Tensor, tb: Tensor, num_graphs: int):
    """ptr offsets of both sides for a graph count, built on the device,
    with the int32 [2] flags that check them (ra_ptr_from_batch)."""
    lib = _lib.load()
    dev = sb.device
    ptr_x = torch.empty(num_graphs + 1, dtype=torch.long, device=dev)
    ptr_y = torch.empty(num_graphs + 1, dtype=torch.long, device=dev)
    flags = torch.empty(2, dtype=torch.int32, device=dev)
    stream = _lib.stream_handle(dev)
    with torch.cuda.device(dev):
        for b, p, k in ((sb, ptr_x, 0), (tb, ptr_y, 1)):
            rc = lib.ra_ptr_from_batch(b.data_ptr(), b.numel(), num_graphs, p.data_ptr(),
                                       flags.data_ptr() + 4 * k, stream)
            _lib.check(rc, "ptr from batch")
    return ptr_x, ptr_y, flags


def pyg_kde_mmd_loss(
    src_pos: Tensor,
    tgt_pos: Tensor,
    *,
    src_batch: Optional[Tensor] = None,
    tgt_batch: Optional[Tensor] = None,
    src_ptr: Optional[Tensor] = None,
    tgt_ptr: Optional[Tensor] = None,
    src_w: Optional[Tensor] = None,
    tgt_w: Optional[Tensor] = None,
    sigma: float = 0.2,
    center: bool = True,
    cosine: bool = False,
    eps: float = 1e-8,
) -> Tuple[Tensor, Tensor, Tensor, Tensor]:
    """KDE/MMD loss for ragged PyG-style batches (rapidalign/kde.py:302-428)."""
    if src_pos.ndim != 2 or tgt_pos.ndim != 2:
        raise ValueError("src_pos and tgt_pos must be 2-D")
    if src_pos.size(1) != tgt_pos.size(1):
        raise ValueError("source and target must share feature dimension")
    if src_pos.device != tgt_pos.device:
        raise ValueError("source and target must be on the same device")
    if isinstance(sigma, Tensor):
        if (sigma <= 0).any():
            raise ValueError("sigma must be positive")
    elif sigma <= 0:
        raise ValueError("sigma must be positive")

    device = src_pos.device
    _lib.require_cuda(src_pos, tgt_pos)
    kw = dict(src_w=src_w, tgt_w=tgt_w, sigma=sigma, center=center, cosine=cosine, eps=eps)

    # both sides as batch vectors: start with the last call's graph count
    # (verified on the device, repeated exactly if wrong), no host round trip
    if (src_ptr is None and tgt_ptr is None and src_batch is not None and
            tgt_batch is not None):
        sb = src_batch.to(device=device, dtype=torch.long).contiguous()
        tb = tgt_batch.to(device=device, dtype=torch.long).contiguous()
        if sb.numel() != src_pos.size(0) or tb.numel() != tgt_pos.size(0):
            raise ValueError("batch length must match number of nodes")
        guess = _GRAPH_COUNT_HINT.get(device.index)
        if guess is not None and sb.numel() > 0 and tb.numel() > 0:
            ptr_x, ptr_y, flags = _batch_ptrs_on_device(sb, tb, guess)
            try:
                return _pyg_segments(src_pos, tgt_pos, ptr_x, ptr_y, guess, False, flags, **kw)
            except GraphCountMismatch:
                pass
        src_batch, tgt_batch = sb, tb

    src_ptr_t, num_src, user_x, tgt_ptr_t, num_tgt, user_y = _ensure_ptrs(
        src_ptr, src_batch, src_pos.size(0), tgt_ptr, tgt_batch, tgt_pos.size(0), device)
    if num_src != num_tgt:
        raise ValueError("source and target batches must have the same length")
    if not (user_x or user_y):
        _GRAPH_COUNT_HINT[device.index] = num_src
    return _pyg_segments(src_pos, tgt_pos, src_ptr_t, tgt_ptr_t, num_src, user_x or user_y,
                         None, **kw)


def _pyg_segments(src_pos, tgt_pos, src_ptr_t, tgt_ptr_t, num_pairs, user_ptr, batch_flags,
                  src_w, tgt_w, sigma, center, cosine, eps):
    """pyg_kde_mmd_loss once the segments are known: ptr offsets of both
    sides (user-given, or built from batch vectors with `batch_flags` still to
    be checked) for `num_pairs` graphs."""
    device = src_pos.device
    dtype = src_pos.dtype
    if num_pairs == 0:
        zero = torch.zeros((0,), device=device, dtype=dtype)
        return zero, zero, zero, zero

    for w, n in ((src_w, src_pos.size(0)), (tgt_w, tgt_pos.size(0))):
        if w is None:
            continue
        if n == 0:
            if w.numel() != 0:
                raise ValueError("weights must be empty when there are no nodes")
        elif w.numel() != n:
            raise ValueError("weights length must equal number of nodes")

    sig, sig_t = _sigma_value(sigma, device)
    spec = Spec(
        layout=_lib.RA_LAYOUT_RAGGED, num_pairs=num_pairs, dim=src_pos.shape[1],
        num_x=src_pos.shape[0], num_y=tgt_pos.shape[0],
        weights_x=_lib.RA_WEIGHTS_SUM if src_w is not None else _lib.RA_WEIGHTS_UNIFORM,
        weights_y=_lib.RA_WEIGHTS_SUM if tgt_w is not None else _lib.RA_WEIGHTS_UNIFORM,
        center=center, sigma=sig, ptr_x=src_ptr_t, ptr_y=tgt_ptr_t,
        check_errors=(user_ptr or src_w is not None or tgt_w is not None),
        batch_flags=batch_flags)
    xw = None if src_w is None else src_w.to(device).reshape(-1)
    yw = None if tgt_w is None else tgt_w.to(device).reshape(-1)
    Kxx, Kyy, Kxy = kde_sums(src_pos, tgt_pos, xw, yw, sig_t, spec)
    return mmd_outputs(Kxx, Kyy, Kxy, cosine, eps, dtype)


def pyg_batch_kde_mmd_loss(src, tgt, *, pos: str = "pos", weight: Optional[str] = None,
                           sigma: float = 0.2, center: bool = True, cosine: bool = False,
                           eps: float = 1e-8) -> Tuple[Tensor, Tensor, Tensor, Tensor]:
    """``pyg_kde_mmd_loss`` on two PyG-style batch objects.

    Takes the point tensors from attribute ``pos`` and optional node weights
    from attribute ``weight`` of ``src`` and ``tgt`` (a
    ``torch_geometric.data.Batch`` or anything with the same attributes).
    The segments come from the batches' ``ptr`` when they carry one -- the
    offsets PyG keeps for every batch, whose checks run on the device with
    no host synchronisation -- else from their sorted ``batch`` vectors
    (kde.py:124-156, one synchronisation for the graph count).
    """
    def field(obj, name):
        if name is None:
            return None
        val = getattr(obj, name, None)
        if val is None:
            raise ValueError(f"batch has no attribute '{name}'")
        return val

    src_pos, tgt_pos = field(src, pos), field(tgt, pos)
    kw = dict(src_w=field(src, weight), tgt_w=field(tgt, weight), sigma=sigma, center=center,
              cosine=cosine, eps=eps)
    s_ptr, t_ptr = getattr(src, "ptr", None), getattr(tgt, "ptr", None)
    if s_ptr is not None and t_ptr is not None:
        return pyg_kde_mmd_loss(src_pos, tgt_pos, src_ptr=s_ptr, tgt_ptr=t_ptr, **kw)
    return pyg_kde_mmd_loss(src_pos, tgt_pos, src_batch=field(src, "batch"),
                            tgt_batch=field(tgt, "batch"), **kw)
