"""The differentiable K-sum operator behind every public entry point.

``kde_sums`` returns ``(Kxx, Kyy, Kxy)`` per pair (float64) for a ragged,
dense or single-pair problem, after the weight normalisation and centering
the caller selects.  Its backward is one epilogue launch over the per-point
sums the fused forward kept in its workspace: the forward evaluates every
unique kernel term once for both the values and the gradients.

Everything runs through the C ABI of ``librapidalign_b200.so``; there is no
CPU path.
"""
from __future__ import annotations

import ctypes
import dataclasses
from dataclasses import dataclass
from typing import Optional, Tuple

import torch

from . import _lib

Tensor = torch.Tensor


@dataclass
class Spec:
    """Problem layout (non-tensor arguments of the autograd Function)."""
    layout: int
    num_pairs: int
    dim: int
    num_x: int
    num_y: int
    nmax_x: int = 0
    nmax_y: int = 0
    weights_x: int = _lib.RA_WEIGHTS_UNIFORM
    weights_y: int = _lib.RA_WEIGHTS_UNIFORM
    center: bool = True
    sigma: float = 0.2
    ptr_x: Optional[Tensor] = None
    ptr_y: Optional[Tensor] = None
    mask_x: Optional[Tensor] = None
    mask_y: Optional[Tensor] = None
    # float64 [P] per-pair bandwidths (then `sigma` is ignored by the kernels
    # and a sigma tensor gets one gradient per pair)
    sigma_pairs: Optional[Tensor] = None
    # which device-detected errors can occur (and must be checked, at the
    # price of one synchronisation): user ptr offsets, SUM-normalised weights
    check_errors: bool = False
    # split evaluation of one problem across a process group (see shard.py)
    shard_index: int = 0
    shard_count: int = 1
    engine: int = 0  # _lib.RA_ENGINE_*: kernel family for dim >= 4 (0 = automatic)
    weight_error_message: str = "weights must sum to a positive value per segment"
    # no weight gradient can be asked for (set by forward_sums): the forward
    # may leave out the per-point sums only grad_wx / grad_wy need
    skip_weight_sums: bool = False
    # int32 [2] device flags of ra_ptr_from_batch for the two sides when ptr_x
    # / ptr_y were built from batch vectors (checked with the error word)
    batch_flags: Optional[Tensor] = None
    # gradients bitwise independent of scheduling (ra_kde_desc.deterministic);
    # None: follow torch.are_deterministic_algorithms_enabled() at the forward
    deterministic: Optional[bool] = None

    def desc(self, need_grad: bool, need_sigma_grad: bool) -> _lib.RaKdeDesc:
        d = _lib.RaKdeDesc()
        d.num_pairs = self.num_pairs
        d.dim = self.dim
        d.layout = self.layout
        d.num_x = self.num_x
        d.num_y = self.num_y
        d.nmax_x = self.nmax_x
        d.nmax_y = self.nmax_y
        d.weights_x = self.weights_x
        d.weights_y = self.weights_y
        d.center = 1 if self.center else 0
        d.need_grad = 1 if need_grad else 0
        d.need_sigma_grad = 1 if need_sigma_grad else 0
        d.shard_index = self.shard_index
        d.shard_count = self.shard_count
        d.sigma = float(self.sigma)
        d.engine = int(self.engine)
        d.skip_weight_sums = 1 if (need_grad and self.skip_weight_sums) else 0
        det = self.deterministic
        if det is None:
            det = torch.are_deterministic_algorithms_enabled()
        d.deterministic = 1 if det else 0
        d.test_hooks = 0
        return d


def _f32(t: Optional[Tensor]) -> Optional[Tensor]:
    if t is None:
        return None
    return t.detach().to(torch.float32).contiguous()


def _inputs(x32, y32, wx32, wy32, spec: Spec) -> _lib.RaKdeInputs:
    i = _lib.RaKdeInputs()
    i.x = _lib.ptr(x32)
    i.y = _lib.ptr(y32)
    i.w_x = _lib.ptr(wx32)
    i.w_y = _lib.ptr(wy32)
    i.ptr_x = _lib.ptr(spec.ptr_x)
    i.ptr_y = _lib.ptr(spec.ptr_y)
    i.mask_x = _lib.ptr(spec.mask_x)
    i.mask_y = _lib.ptr(spec.mask_y)
    i.sigma_pairs = _lib.ptr(spec.sigma_pairs)
    return i


class GraphCountMismatch(Exception):
    """The graph count a batch-vector call was launched with is not the one
    its batch vectors hold (raised before any result is returned; the caller
    repeats the call with the exact count)."""


def _raise_batch_flags(flags) -> None:
    if any(f & _lib.RA_BATCH_UNSORTED for f in flags):
        raise ValueError("batch indices must be sorted for contiguous blocks")
    if any(f & _lib.RA_BATCH_NEGATIVE for f in flags):
        raise ValueError("batch indices must be non-negative")
    if any(f & _lib.RA_BATCH_COUNT for f in flags):
        raise GraphCountMismatch()


def uses_tensor_cores(spec: Spec) -> bool:
    """Whether the forward runs the tensor-core kernels (padded dim 32, 64 or
    128 on the automatic or tensor engine), whose bounded waits can expire."""
    if spec.dim <= 3 or spec.engine == _lib.RA_ENGINE_SIMT:
        return False
    return _wide(spec)


def _wide(spec: Spec) -> bool:
    """Padded dim 32, 64 or 128: the O(N) passes may stream their rows by bulk
    copies (equal weights, no mask), whose bounded waits can expire too."""
    if spec.dim <= 3:
        return False
    dp = 4
    while dp < spec.dim:
        dp <<= 1
    return dp in (32, 64, 128)


# error words of finished backward passes, read once their copies are done
# (at the next forward or backward): a backward returns without stopping the
# GPU, and an expired wait in it still raises, one call later
_LATE_WORDS: list = []


def _check_late(lib) -> None:
    keep = []
    failed = None
    for w in _LATE_WORDS:
        if w.event.query():
            code = lib.ra_kde_status_of_error_word(w.read()[0])
            if code != _lib.RA_OK and failed is None:
                failed = code
        else:
            keep.append(w)
    _LATE_WORDS[:] = keep
    if failed is not None:
        _lib.check(failed, "kde backward (an earlier call)")


_READ_STREAMS: dict = {}


def _read_stream(device):
    """A side stream per device for small device-to-host reads, with its raw
    handle: a read enqueued there waits for its data (an event), but the
    kernels enqueued after it on the compute stream do not wait for the read
    -- which may queue behind a large host-to-device copy on the copy
    engines."""
    s = _READ_STREAMS.get(device.index)
    if s is None:
        st = torch.cuda.Stream(device)
        s = _READ_STREAMS[device.index] = (st, st.cuda_stream)
    return s


_PINNED_WORDS: list = []  # page-locked int32 [16] buffers of finished reads
_WORDS_MAX = 16


def _mark(stream) -> torch.cuda.Event:
    """An event at the current end of `stream` (what a later read waits for)."""
    ev = torch.cuda.Event()
    ev.record(stream)
    return ev


class _ErrorWord:
    """An asynchronous read of the workspace's error word (and, optionally,
    of batch flags): copied into pinned host memory on a side stream once the
    compute stream has passed `ready` (an event), and waited for through an
    event, so the host stops only when it needs the answer while later kernels
    keep the GPU busy.  Created after the kernels that follow `ready` are
    enqueued, so they do not wait for the host to set up the read.  The
    caller keeps `ws` and `flags` alive until read() returns."""

    def __init__(self, ws: Tensor, ready: torch.cuda.Event, flags: Optional[Tensor] = None):
        self.n = 1 + (0 if flags is None else flags.numel())
        if self.n > _WORDS_MAX:
            raise RuntimeError("too many flags for an error-word read")
        try:
            self.host = _PINNED_WORDS.pop()
        except IndexError:
            self.host = torch.empty(_WORDS_MAX, dtype=torch.int32, pin_memory=True)
        side, handle = _read_stream(ws.device)
        side.wait_event(ready)
        rc = _lib.load().ra_kde_error_word_async(
            ws.data_ptr(), None if flags is None else flags.data_ptr(), self.n - 1,
            self.host.data_ptr(), handle)
        _lib.check(rc, "error word read")
        self.event = torch.cuda.Event()
        self.event.record(side)

    def read(self):
        self.event.synchronize()
        words = self.host[:self.n].tolist()
        _PINNED_WORDS.append(self.host)  # the copies are done: reusable
        self.host = None
        return words


def _raise_data_error(code: int, spec: Spec) -> None:
    if code == _lib.RA_OK:
        return
    if code == _lib.RA_ERR_PTR_START:
        raise ValueError("ptr must start at 0")
    if code == _lib.RA_ERR_PTR_END:
        raise ValueError("ptr[-1] must equal number of nodes")
    if code == _lib.RA_ERR_PTR_ORDER:
        raise ValueError("ptr offsets must match node stacks")
    if code == _lib.RA_ERR_WEIGHT_SUM:
        raise ValueError(spec.weight_error_message)
    _lib.check(code, "kde forward")


class _State:
    """What a backward needs from its forward: the fp32 inputs, the workspace
    holding the per-point sums, and the original dtypes/shapes."""

    def __init__(self, spec, need_sigma_grad, keep, meta, pending=None):
        self.spec = spec
        self.need_sigma_grad = need_sigma_grad
        self.keep = keep
        self.meta = meta
        self.pending = pending  # error word read after the tile kernels (tensor cores)


def partial_buffers(lib, desc, ws: Tensor) -> Tuple[Tensor, Optional[Tensor]]:
    """Views of the two workspace regions a split evaluation sums across its
    group: the fp64 item partials and the fp32 per-point sums (or None)."""
    f64, n64 = ctypes.c_void_p(), ctypes.c_size_t()
    f32, n32 = ctypes.c_void_p(), ctypes.c_size_t()
    rc = lib.ra_kde_partials(ctypes.byref(desc), ws.data_ptr(), ws.numel(), ctypes.byref(f64),
                             ctypes.byref(n64), ctypes.byref(f32), ctypes.byref(n32))
    _lib.check(rc, "kde partials")
    base = ws.data_ptr()
    o64 = f64.value - base
    t64 = ws[o64:o64 + 8 * n64.value].view(torch.float64)
    t32 = None
    if n32.value:
        o32 = f32.value - base
        t32 = ws[o32:o32 + 4 * n32.value].view(torch.float32)
    return t64, t32


def forward_sums(x: Tensor, y: Tensor, w_x: Optional[Tensor], w_y: Optional[Tensor],
                 sigma_t: Optional[Tensor], spec: Spec, need_grad: bool, reduce=None):
    """Run the fused forward; returns (K float64 [3P], state or None).

    With spec.shard_count > 1 the forward evaluates this shard's work items
    only; `reduce(f64_view, f32_view)` must then sum the partial buffers
    across the group in place before K is formed."""
    lib = _lib.load()
    if _LATE_WORDS:
        _check_late(lib)
    device = x.device
    need_sigma_grad = need_grad and sigma_t is not None and sigma_t.requires_grad
    weights_grad = any(w is not None and w.requires_grad for w in (w_x, w_y))
    if need_grad and not weights_grad and not spec.skip_weight_sums:
        spec = dataclasses.replace(spec, skip_weight_sums=True)
    if spec.deterministic is None:  # fixed now, so that the backward matches
        spec = dataclasses.replace(spec,
                                   deterministic=torch.are_deterministic_algorithms_enabled())
    x32, y32 = _f32(x), _f32(y)
    wx32, wy32 = _f32(w_x), _f32(w_y)
    desc = spec.desc(need_grad, need_sigma_grad)
    inp = _inputs(x32, y32, wx32, wy32, spec)
    nbytes = lib.ra_kde_workspace_bytes(ctypes.byref(desc))
    if nbytes == 0:
        raise RuntimeError("rapidalign_b200: invalid problem description")
    ws = _lib.workspace(nbytes, device)
    K = torch.empty(3 * spec.num_pairs, dtype=torch.float64, device=device)
    tstream = torch.cuda.current_stream(device)
    stream = tstream.cuda_stream
    pending = None
    with torch.cuda.device(device):
        rc = lib.ra_kde_forward_prepare(ctypes.byref(desc), ctypes.byref(inp), ws.data_ptr(),
                                        ws.numel(), stream)
        _lib.check(rc, "kde forward")
        # the data errors are known once the preparation ran: read them while
        # the tile kernels run, instead of stopping the GPU to ask
        prepared = None
        if spec.check_errors or spec.batch_flags is not None:
            prepared = _mark(tstream)
        rc = lib.ra_kde_forward_compute(ctypes.byref(desc), ctypes.byref(inp), K.data_ptr(),
                                        ws.data_ptr(), ws.numel(), stream)
        _lib.check(rc, "kde forward")
        early = None if prepared is None else _ErrorWord(ws, prepared, spec.batch_flags)
        if _wide(spec):
            pending = _ErrorWord(ws, _mark(tstream))  # an expired wait shows after the tiles
        if early is not None:
            words = early.read()
            if len(words) > 1:
                _raise_batch_flags(words[1:])
            if spec.check_errors:
                _raise_data_error(lib.ra_kde_status_of_error_word(words[0]), spec)
        if spec.shard_count > 1:
            if reduce is None:
                raise RuntimeError("a split evaluation needs a reduction of its partials")
            reduce(*partial_buffers(lib, desc, ws))
            rc = lib.ra_kde_forward_finish(ctypes.byref(desc), K.data_ptr(), ws.data_ptr(),
                                           ws.numel(), stream)
            _lib.check(rc, "kde forward finish")
        if pending is not None and not need_grad:
            _check_pending(lib, pending)
            pending = None
    state = None
    if need_grad:
        state = _State(spec, need_sigma_grad,
                       (x32, y32, wx32, wy32, ws, spec.ptr_x, spec.ptr_y, spec.mask_x,
                        spec.mask_y),
                       (x.dtype, x.shape, y.dtype, y.shape,
                        None if w_x is None else (w_x.dtype, w_x.shape),
                        None if w_y is None else (w_y.dtype, w_y.shape),
                        None if sigma_t is None else (sigma_t.dtype, sigma_t.shape)),
                       pending)
    return K, state


def _check_pending(lib, pending: _ErrorWord) -> None:
    code = lib.ra_kde_status_of_error_word(pending.read()[0])
    if code != _lib.RA_OK:
        _lib.check(code, "kde forward (tensor-core kernels)")


def backward_sums(state: _State, coef: Tensor, need) -> tuple:
    """Gradients (x, y, w_x, w_y, sigma) for coefficients coef = dL/d(Kxx|Kyy|Kxy)
    (float64 [3P]); `need` flags which of the five are wanted."""
    lib = _lib.load()
    if _LATE_WORDS:
        _check_late(lib)
    spec = state.spec
    x32, y32, wx32, wy32, ws = state.keep[:5]
    device = x32.device
    P = spec.num_pairs
    coef = coef.to(device=device, dtype=torch.float64).contiguous()
    nx = x32.shape[0] if x32.dim() == 2 else x32.shape[0] * x32.shape[1]
    ny = y32.shape[0] if y32.dim() == 2 else y32.shape[0] * y32.shape[1]
    gx = torch.empty_like(x32) if need[0] else None
    gy = torch.empty_like(y32) if need[1] else None
    gwx = (torch.empty(nx, dtype=torch.float64, device=device)
           if (need[2] and wx32 is not None) else None)
    gwy = (torch.empty(ny, dtype=torch.float64, device=device)
           if (need[3] and wy32 is not None) else None)
    gsig = (torch.empty(P, dtype=torch.float64, device=device)
            if (need[4] and state.need_sigma_grad) else None)
    grads = _lib.RaKdeGrads()
    grads.grad_x = _lib.ptr(gx)
    grads.grad_y = _lib.ptr(gy)
    grads.grad_wx = _lib.ptr(gwx)
    grads.grad_wy = _lib.ptr(gwy)
    grads.grad_sigma = _lib.ptr(gsig)
    desc = spec.desc(True, state.need_sigma_grad)
    inp = _inputs(x32, y32, wx32, wy32, spec)
    with torch.cuda.device(device):
        rc = lib.ra_kde_backward(ctypes.byref(desc), ctypes.byref(inp), coef.data_ptr(),
                                 ctypes.byref(grads), ws.data_ptr(), ws.numel(),
                                 _lib.stream_handle(device))
    _lib.check(rc, "kde backward")
    if _wide(spec):
        # the backward's own bounded waits: its error word, read later
        word = _ErrorWord(ws, _mark(torch.cuda.current_stream(device)))
        ws.record_stream(_read_stream(device)[0])  # not reused before the copy
        _LATE_WORDS.append(word)
    if state.pending is not None:
        # the forward's tile kernels are done by the time this returns, while
        # the backward just enqueued keeps the GPU busy
        pending, state.pending = state.pending, None
        _check_pending(lib, pending)
    xdt, xsh, ydt, ysh, wxm, wym, sm = state.meta
    out_x = gx.to(xdt).reshape(xsh) if gx is not None else None
    out_y = gy.to(ydt).reshape(ysh) if gy is not None else None
    out_wx = gwx.to(wxm[0]).reshape(wxm[1]) if gwx is not None else None
    out_wy = gwy.to(wym[0]).reshape(wym[1]) if gwy is not None else None
    if gsig is None:
        out_s = None
    elif spec.sigma_pairs is not None:  # one bandwidth per pair
        out_s = gsig.to(sm[0]).reshape(sm[1])
    else:
        out_s = gsig.sum().to(sm[0]).reshape(sm[1])
    return out_x, out_y, out_wx, out_wy, out_s


def needs_grad(*tensors) -> bool:
    return torch.is_grad_enabled() and any(
        t is not None and isinstance(t, Tensor) and t.requires_grad for t in tensors)


class KDESums(torch.autograd.Function):
    """(x, y, w_x, w_y, sigma) -> (Kxx, Kyy, Kxy), all float64 of shape (P,)."""

    @staticmethod
    def forward(ctx, x: Tensor, y: Tensor, w_x: Optional[Tensor], w_y: Optional[Tensor],
                sigma_t: Optional[Tensor], spec: Spec, need_grad: bool, reduce=None):
        K, state = forward_sums(x, y, w_x, w_y, sigma_t, spec, need_grad, reduce)
        ctx.state = state
        P = spec.num_pairs
        return K[:P], K[P:2 * P], K[2 * P:]

    @staticmethod
    def backward(ctx, gKxx: Optional[Tensor], gKyy: Optional[Tensor], gKxy: Optional[Tensor]):
        state = ctx.state
        if state is None:
            return None, None, None, None, None, None, None, None
        P = state.spec.num_pairs
        device = state.keep[0].device

        def g_or_zero(g):
            if g is None:
                return torch.zeros(P, dtype=torch.float64, device=device)
            return g.to(torch.float64)

        coef = _adjacent(gKxx, gKyy, gKxy, P)
        if coef is None:
            coef = torch.cat([g_or_zero(gKxx), g_or_zero(gKyy), g_or_zero(gKxy)])
        grads = backward_sums(state, coef, ctx.needs_input_grad[:5])
        return grads + (None, None, None)


def _adjacent(a: Optional[Tensor], b: Optional[Tensor], c: Optional[Tensor],
              P: int) -> Optional[Tensor]:
    """The float64 [3P] buffer whose thirds a, b, c are, when they are (no copy
    needed), else None."""
    if a is None or b is None or c is None or P == 0:
        return None
    for t in (a, b, c):
        if t.dtype != torch.float64 or not t.is_contiguous() or t.numel() != P:
            return None
    if (a.untyped_storage().data_ptr() != b.untyped_storage().data_ptr() or
            a.untyped_storage().data_ptr() != c.untyped_storage().data_ptr()):
        return None
    if b.data_ptr() != a.data_ptr() + 8 * P or c.data_ptr() != a.data_ptr() + 16 * P:
        return None
    return a.as_strided((3 * P,), (1,), a.storage_offset())


class MMDOutputs(torch.autograd.Function):
    """(Kxx, Kyy, Kxy) float64 (P,) -> (loss, Kxx, Kyy, Kxy) as float32 or
    float64, in one launch (ra_mmd_outputs); the backward writes dL/dK for
    KDESums in one launch (ra_mmd_outputs_backward).  The loss is that of
    rapidalign/kde.py:103-107 (or the cosine form), in float64."""

    @staticmethod
    def forward(ctx, Kxx: Tensor, Kyy: Tensor, Kxy: Tensor, cosine: bool, eps: float,
                f64: bool):
        lib = _lib.load()
        P = Kxx.numel()
        K = _adjacent(Kxx, Kyy, Kxy, P)
        if K is None:
            K = torch.cat([Kxx.reshape(-1), Kyy.reshape(-1), Kxy.reshape(-1)]).to(torch.float64)
        odt = torch.float64 if f64 else torch.float32
        outs = [torch.empty(P, dtype=odt, device=K.device) for _ in range(4)]
        with torch.cuda.device(K.device):
            rc = lib.ra_mmd_outputs(K.data_ptr() if P else None, P, int(bool(cosine)),
                                    float(eps), int(f64), *[_lib.ptr(o) for o in outs],
                                    _lib.stream_handle(K.device))
        _lib.check(rc, "mmd outputs")
        ctx.save_for_backward(K)
        ctx.cosine, ctx.eps, ctx.f64, ctx.odt = bool(cosine), float(eps), bool(f64), odt
        # an output without a gradient stays None (a null pointer, read as zero)
        # instead of a zero tensor filled on the device
        ctx.set_materialize_grads(False)
        return tuple(outs)

    @staticmethod
    def backward(ctx, gl, ga, gb, gc):
        lib = _lib.load()
        K, = ctx.saved_tensors
        P = K.numel() // 3
        gs = [None if g is None else g.to(ctx.odt).contiguous() for g in (gl, ga, gb, gc)]
        coef = torch.empty(3 * P, dtype=torch.float64, device=K.device)
        with torch.cuda.device(K.device):
            rc = lib.ra_mmd_outputs_backward(K.data_ptr() if P else None, P, int(ctx.cosine),
                                             ctx.eps, int(ctx.f64), *[_lib.ptr(g) for g in gs],
                                             _lib.ptr(coef), _lib.stream_handle(K.device))
        _lib.check(rc, "mmd outputs backward")
        return coef[:P], coef[P:2 * P], coef[2 * P:], None, None, None


def mmd_outputs(Kxx: Tensor, Kyy: Tensor, Kxy: Tensor, cosine: bool, eps: float,
                dtype: torch.dtype) -> Tuple[Tensor, Tensor, Tensor, Tensor]:
    """(loss, Kxx, Kyy, Kxy) in `dtype` from the float64 sums (one launch for
    float32 or float64 outputs; other dtypes are rounded once from float64)."""
    if dtype in (torch.float32, torch.float64):
        return MMDOutputs.apply(Kxx, Kyy, Kxy, cosine, eps, dtype == torch.float64)
    outs = MMDOutputs.apply(Kxx, Kyy, Kxy, cosine, eps, True)
    return tuple(o.to(dtype) for o in outs)


def kde_sums(x: Tensor, y: Tensor, w_x: Optional[Tensor], w_y: Optional[Tensor],
             sigma_t: Optional[Tensor], spec: Spec, reduce=None) -> Tuple[Tensor, Tensor, Tensor]:
    need = needs_grad(x, y, w_x, w_y, sigma_t)
    return KDESums.apply(x, y, w_x, w_y, sigma_t, spec, need, reduce)
