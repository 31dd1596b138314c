"""The C-ABI library loads and exports every function include/rapidalign_b200.h
declares (no compute: no GPU needed)."""
import ctypes
import os
import re

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "rapidalign_b200.h")


def declared_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^RA_API [^(]*?\b(ra_\w+)\(", text, flags=re.M)))


@pytest.fixture(scope="module")
def lib():
    from rapidalign_b200 import build as b
    path = b.build()
    return ctypes.CDLL(path)


def test_header_declares_entry_points():
    names = declared_functions()
    for must in ("ra_kde_mmd_forward", "ra_kde_mmd_forward_segmented",
                 "ra_kde_mmd_backward_segmented", "ra_kde_forward", "ra_kde_backward"):
        assert must in names


def test_library_exports_every_declared_symbol(lib):
    for name in declared_functions():
        assert hasattr(lib, name), name


def test_python_binding_covers_header(lib):
    from rapidalign_b200 import _lib
    assert set(_lib.SIGNATURES) == set(declared_functions())


def test_host_side_calls_without_gpu(lib):
    """Pure host functions: status strings and workspace sizing."""
    from rapidalign_b200 import _lib
    L = _lib.load()
    assert L.ra_status_string(0) == b"ok"
    assert b"sigma" in L.ra_status_string(2)
    d = _lib.RaKdeDesc(num_pairs=4, dim=3, layout=0, num_x=100, num_y=120, weights_x=3,
                       weights_y=3, center=1, need_grad=1, sigma=0.25)
    n = L.ra_kde_workspace_bytes(ctypes.byref(d))
    assert n > 0 and n % 256 == 0
    d.dim = 0
    assert L.ra_kde_workspace_bytes(ctypes.byref(d)) == 0
    assert L.ra_kde_mmd_forward_segmented_workspace_bytes(4, 100, 120, 3) > 0
    # invalid arguments are rejected before anything touches a device
    rc = L.ra_kde_forward(None, None, None, None, 0, None)
    assert rc == _lib.RA_ERR_INVALID_ARGUMENT


def test_error_word_decoding(lib):
    """The status each device error bit stands for (ra_kde_status_of_error_word),
    the same mapping ra_kde_check applies after reading the word back."""
    from rapidalign_b200 import _lib
    L = _lib.load()
    assert L.ra_kde_status_of_error_word(0) == _lib.RA_OK
    assert L.ra_kde_status_of_error_word(1) == _lib.RA_ERR_PTR_START
    assert L.ra_kde_status_of_error_word(2) == _lib.RA_ERR_PTR_END
    assert L.ra_kde_status_of_error_word(4) == _lib.RA_ERR_PTR_ORDER
    assert L.ra_kde_status_of_error_word(8) == _lib.RA_ERR_WEIGHT_SUM
    assert L.ra_kde_status_of_error_word(16) == _lib.RA_ERR_DEVICE_TIMEOUT
    assert L.ra_kde_status_of_error_word(32) == _lib.RA_ERR_SIGMA
    assert L.ra_kde_status_of_error_word(2 | 16) == _lib.RA_ERR_PTR_END  # ptr errors first


def test_test_hooks_are_validated(lib):
    from rapidalign_b200 import _lib
    L = _lib.load()
    d = _lib.RaKdeDesc(num_pairs=2, dim=32, layout=0, num_x=100, num_y=120, weights_x=3,
                       weights_y=3, need_grad=1, sigma=1.0, test_hooks=_lib.RA_TEST_NO_MMA)
    assert L.ra_kde_workspace_bytes(ctypes.byref(d)) > 0
    d.test_hooks = 4  # not a hook
    assert L.ra_kde_workspace_bytes(ctypes.byref(d)) == 0
