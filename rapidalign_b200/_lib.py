"""ctypes binding of ``librapidalign_b200.so`` (the C ABI in
``include/rapidalign_b200.h``) plus the torch-side plumbing: current stream,
workspace allocation and status-code to exception mapping.

The library is built in-tree by ``rapidalign_b200/build.py``.  There is no
fallback: if the shared library is missing or fails to load, every CUDA entry
point raises.
"""
from __future__ import annotations

import ctypes
import os
import threading
from typing import Optional

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "librapidalign_b200.so")

# enum values (include/rapidalign_b200.h)
RA_OK = 0
RA_ERR_INVALID_ARGUMENT = 1
RA_ERR_SIGMA = 2
RA_ERR_WORKSPACE = 3
RA_ERR_CUDA = 4
RA_ERR_PTR_START = 16
RA_ERR_PTR_END = 17
RA_ERR_PTR_ORDER = 18
RA_ERR_WEIGHT_SUM = 19
RA_ERR_STATE = 20
RA_ERR_SCRATCH_LIMIT = 21
RA_ERR_DEVICE_TIMEOUT = 22

RA_LAYOUT_RAGGED = 0
RA_LAYOUT_DENSE = 1

RA_WEIGHTS_RAW = 0
RA_WEIGHTS_SUM = 1
RA_WEIGHTS_SUM_CLAMPED = 2
RA_WEIGHTS_UNIFORM = 3

RA_ENGINE_AUTO = 0
RA_ENGINE_SIMT = 1
RA_ENGINE_TENSOR = 2

RA_TEST_NO_MMA = 1
RA_TEST_RING_IDLE = 2

RA_BATCH_UNSORTED = 1
RA_BATCH_NEGATIVE = 2
RA_BATCH_COUNT = 4


class RaKdeDesc(ctypes.Structure):
    _fields_ = [
        ("num_pairs", ctypes.c_int64),
        ("dim", ctypes.c_int32),
        ("layout", ctypes.c_int32),
        ("num_x", ctypes.c_int64),
        ("num_y", ctypes.c_int64),
        ("nmax_x", ctypes.c_int64),
        ("nmax_y", ctypes.c_int64),
        ("weights_x", ctypes.c_int32),
        ("weights_y", ctypes.c_int32),
        ("center", ctypes.c_int32),
        ("need_grad", ctypes.c_int32),
        ("need_sigma_grad", ctypes.c_int32),
        ("shard_index", ctypes.c_int32),
        ("shard_count", ctypes.c_int32),
        ("sigma", ctypes.c_double),
        ("engine", ctypes.c_int32),
        ("skip_weight_sums", ctypes.c_int32),
        ("deterministic", ctypes.c_int32),
        ("test_hooks", ctypes.c_int32),
    ]


class RaPdlCloud(ctypes.Structure):
    _fields_ = [
        ("points", ctypes.c_void_p),
        ("perm", ctypes.c_void_p),
        ("ptr", ctypes.c_void_p),
        ("pair_offsets", ctypes.c_void_p),
        ("num_pairs", ctypes.c_int64),
        ("max_group", ctypes.c_int64),
    ]


class RaKdeInputs(ctypes.Structure):
    _fields_ = [
        ("x", ctypes.c_void_p),
        ("y", ctypes.c_void_p),
        ("w_x", ctypes.c_void_p),
        ("w_y", ctypes.c_void_p),
        ("ptr_x", ctypes.c_void_p),
        ("ptr_y", ctypes.c_void_p),
        ("mask_x", ctypes.c_void_p),
        ("mask_y", ctypes.c_void_p),
        ("sigma_pairs", ctypes.c_void_p),
    ]


class RaKdeGrads(ctypes.Structure):
    _fields_ = [
        ("grad_x", ctypes.c_void_p),
        ("grad_y", ctypes.c_void_p),
        ("grad_wx", ctypes.c_void_p),
        ("grad_wy", ctypes.c_void_p),
        ("grad_sigma", ctypes.c_void_p),
    ]


# Every symbol the header declares, with (restype, argtypes).
_V = ctypes.c_void_p
_I64 = ctypes.c_int64
_I32 = ctypes.c_int32
_D = ctypes.c_double
_SZ = ctypes.c_size_t
SIGNATURES = {
    "ra_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "ra_kde_workspace_bytes": (_SZ, [ctypes.POINTER(RaKdeDesc)]),
    "ra_kde_forward": (ctypes.c_int, [ctypes.POINTER(RaKdeDesc), ctypes.POINTER(RaKdeInputs),
                                      _V, _V, _SZ, _V]),
    "ra_kde_forward_prepare": (ctypes.c_int, [ctypes.POINTER(RaKdeDesc),
                                              ctypes.POINTER(RaKdeInputs), _V, _SZ, _V]),
    "ra_kde_forward_compute": (ctypes.c_int, [ctypes.POINTER(RaKdeDesc),
                                              ctypes.POINTER(RaKdeInputs), _V, _V, _SZ, _V]),
    "ra_ptr_from_batch": (ctypes.c_int, [_V, _I64, _I64, _V, _V, _V]),
    "ra_kde_backward": (ctypes.c_int, [ctypes.POINTER(RaKdeDesc), ctypes.POINTER(RaKdeInputs),
                                       _V, ctypes.POINTER(RaKdeGrads), _V, _SZ, _V]),
    "ra_kde_check": (ctypes.c_int, [_V, _V]),
    "ra_kde_status_of_error_word": (ctypes.c_int, [ctypes.c_int]),
    "ra_kde_error_word_async": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32,
                                               ctypes.c_void_p, ctypes.c_void_p]),
    "ra_mmd_outputs": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int,
                                      ctypes.c_double, ctypes.c_int, ctypes.c_void_p,
                                      ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                      ctypes.c_void_p]),
    "ra_mmd_outputs_backward": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int,
                                               ctypes.c_double, ctypes.c_int, ctypes.c_void_p,
                                               ctypes.c_void_p, ctypes.c_void_p,
                                               ctypes.c_void_p, ctypes.c_void_p,
                                               ctypes.c_void_p]),
    "ra_kde_check_noalloc": (ctypes.c_int, [_V]),
    "ra_kde_partials": (ctypes.c_int, [ctypes.POINTER(RaKdeDesc), _V, _SZ,
                                       ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(_SZ),
                                       ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(_SZ)]),
    "ra_kde_forward_finish": (ctypes.c_int, [ctypes.POINTER(RaKdeDesc), _V, _V, _SZ, _V]),
    "ra_kde_forward_profiled": (ctypes.c_int, [ctypes.POINTER(RaKdeDesc),
                                               ctypes.POINTER(RaKdeInputs), _V, _V, _SZ, _V,
                                               ctypes.POINTER(ctypes.c_float)]),
    "ra_kde_mmd_forward_workspace_bytes": (_SZ, [_I64, _I64, _I64, _I32]),
    "ra_kde_mmd_forward": (ctypes.c_int, [_V, _V, _V, _V, _V, _V, _I64, _I64, _I64, _I32, _D,
                                          _V, _V, _V, _V, _SZ, _V]),
    "ra_kde_mmd_forward_segmented_workspace_bytes": (_SZ, [_I64, _I64, _I64, _I32]),
    "ra_kde_mmd_forward_segmented": (ctypes.c_int, [_V, _V, _V, _V, _V, _V, _I64, _I64, _I64,
                                                    _I32, _D, _V, _V, _V, _V, _SZ, _V]),
    "ra_kde_mmd_backward_segmented_workspace_bytes": (_SZ, [_I64, _I64, _I64, _I32]),
    "ra_kde_mmd_backward_segmented": (ctypes.c_int, [_V, _V, _V, _V, _V, _V, _I64, _I64, _I64,
                                                     _I32, _V, _D, _V, _V, _V, _V, _V, _V, _SZ,
                                                     _V]),
    "ra_kde_mmd_forward_segmented_noalloc": (ctypes.c_int, [_V, _V, _V, _V, _V, _V, _I64, _I64,
                                                            _I64, _I32, _D, _V, _V, _V, _V]),
    "ra_kde_exact_workspace_bytes": (_SZ, [_I64, _I64]),
    "ra_kde_exact_f64": (ctypes.c_int, [_V, _V, _V, _V, _V, _V, _I64, _I64, _I64, _I32, _D,
                                        _V, _V, _V, _V, _V, _V, _V, _V, _V, _V, _SZ, _V]),
    "ra_kde_exact_matrices_f64": (ctypes.c_int, [_V, _I64, _V, _I64, _I32, _D, _V, _V, _V]),
    "ra_pdl_workspace_bytes": (_SZ, [_I64, _I64, _I64]),
    "ra_pdl_forward": (ctypes.c_int, [ctypes.POINTER(RaPdlCloud), ctypes.POINTER(RaPdlCloud),
                                      _I64, _I32, _V, _V, _SZ, _V]),
    "ra_pdl_backward": (ctypes.c_int, [ctypes.POINTER(RaPdlCloud), ctypes.POINTER(RaPdlCloud),
                                       _I64, _I32, _V, _V, _V, _V, _SZ, _V]),
    "ra_kernel_launch_count": (ctypes.c_ulonglong, []),
    "ra_probe_fp32_peak": (ctypes.c_int, [_V, _I64, ctypes.c_int, ctypes.POINTER(_D), _V]),
}

_lib = None
_lock = threading.Lock()


def load(path: Optional[str] = None):
    """Load (once) and return the shared library; raises if it is missing."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = path or LIB_PATH
        if not os.path.exists(p):
            raise RuntimeError(
                f"rapidalign_b200: CUDA library not built ({p} missing); run "
                "`python -m rapidalign_b200.build` or __graft_entry__.build()")
        lib = ctypes.CDLL(p)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if path is None:
            _lib = lib
        return lib


def status_string(code: int) -> str:
    return load().ra_status_string(int(code)).decode()


def check(code: int, what: str = "") -> None:
    if code != RA_OK:
        msg = status_string(code)
        if code in (RA_ERR_SIGMA,):
            raise ValueError("sigma must be positive")
        raise RuntimeError(f"rapidalign_b200{': ' + what if what else ''}: {msg} (status {code})")


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    """A 256-byte aligned uint8 device buffer of at least nbytes."""
    buf = torch.empty(max(int(nbytes), 1) + 256, dtype=torch.uint8, device=device)
    off = (-buf.data_ptr()) % 256
    return buf[off:off + max(int(nbytes), 1)]


def launch_count() -> int:
    return int(load().ra_kernel_launch_count())


def require_cuda(*tensors: Optional[torch.Tensor]) -> torch.device:
    """The product path runs on CUDA only: fail loudly otherwise."""
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError(
                "rapidalign_b200 computes on CUDA devices only (got a tensor on "
                f"{t.device}); move the inputs to a CUDA device")
        if dev is None:
            dev = t.device
    if dev is None:
        raise RuntimeError("rapidalign_b200: no CUDA tensor given")
    load()
    return dev
