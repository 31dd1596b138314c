"""Host-side behaviour of the public API that needs no GPU: the reference's
argument errors (same ValueError messages, rapidalign/kde.py and
autograd_kde.py) and the loud failure of the product path on CPU tensors."""
import pytest
import torch

import rapidalign_b200 as ra


def test_kde_mmd_loss_shape_errors():
    with pytest.raises(ValueError, match="x and y must be"):
        ra.kde_mmd_loss(torch.randn(5, 3), torch.randn(5, 2))
    with pytest.raises(ValueError, match="x and y must be"):
        ra.kde_mmd_loss(torch.randn(5), torch.randn(5, 3))
    with pytest.raises(ValueError, match="sigma must be positive"):
        ra.kde_mmd_loss(torch.randn(5, 3), torch.randn(5, 3), sigma=0.0)
    with pytest.raises(ValueError, match="sigma must be positive"):
        ra.kde_mmd_loss(torch.randn(5, 3), torch.randn(5, 3), sigma=torch.tensor(-1.0))


def test_dense_errors():
    x = torch.randn(2, 4, 3)
    m = torch.ones(2, 4, dtype=torch.bool)
    with pytest.raises(ValueError, match="sigma must be positive"):
        ra.kde_mmd_loss_dense(x, x, m, m, sigma=-0.1)
    with pytest.raises(ValueError, match=r"x and y must have shape \(B, Nmax, D\)"):
        ra.kde_mmd_loss_dense(x, torch.randn(3, 4, 3), m, m)


def test_pyg_errors():
    x = torch.randn(6, 3)
    with pytest.raises(ValueError, match="must be 2-D"):
        ra.pyg_kde_mmd_loss(torch.randn(6), x, src_ptr=torch.tensor([0, 6]),
                            tgt_ptr=torch.tensor([0, 6]))
    with pytest.raises(ValueError, match="share feature dimension"):
        ra.pyg_kde_mmd_loss(x, torch.randn(6, 2), src_ptr=torch.tensor([0, 6]),
                            tgt_ptr=torch.tensor([0, 6]))
    with pytest.raises(ValueError, match="sigma must be positive"):
        ra.pyg_kde_mmd_loss(x, x, src_ptr=torch.tensor([0, 6]), tgt_ptr=torch.tensor([0, 6]),
                            sigma=0)


def test_segmented_sigma_must_be_scalar():
    x = torch.randn(4, 3)
    w = torch.ones(4)
    p = torch.tensor([0, 4])
    with pytest.raises(ValueError, match="sigma must be a scalar tensor"):
        ra.segmented_kde_loss(x, x, w, w, p, p, torch.tensor([0.3]))


def test_cpu_tensors_fail_loudly():
    """No CPU fallback: the product path refuses host tensors."""
    x = torch.randn(8, 3)
    with pytest.raises(RuntimeError, match="CUDA devices only"):
        ra.kde_mmd_loss(x, x)
    with pytest.raises(RuntimeError, match="CUDA devices only"):
        ra.pyg_kde_mmd_loss(x, x, src_ptr=torch.tensor([0, 8]), tgt_ptr=torch.tensor([0, 8]))
    m = torch.ones(1, 8, dtype=torch.bool)
    with pytest.raises(RuntimeError, match="CUDA devices only"):
        ra.kde_mmd_loss_dense(x[None], x[None], m, m)
    w = torch.ones(8)
    p = torch.tensor([0, 8])
    with pytest.raises(RuntimeError, match="CUDA devices only"):
        ra.segmented_kde_loss(x, x, w, w, p, p, torch.tensor(0.3))


def test_legacy_ops_check_device():
    from rapidalign_b200 import _cuda
    x = torch.randn(8, 3)
    w = torch.ones(8)
    p = torch.tensor([0, 8])
    with pytest.raises(RuntimeError, match="must be CUDA tensor"):
        _cuda.kde_mmd_forward_segmented(x, x, w, w, p, p, 0.2)
    with pytest.raises(RuntimeError, match="must be CUDA tensor"):
        _cuda.kde_mmd_forward(x[None], x[None], w[None], w[None], w[None].bool(),
                              w[None].bool(), 0.2)


def test_backward_error_words_are_read_at_the_next_call():
    """A backward returns without stopping the GPU; the copy of its error word
    is read at the next forward or backward: a finished clean word is
    dropped, an unfinished one kept, a finished word with the timeout bit
    raises (stand-in words, no GPU)."""
    from rapidalign_b200 import _core, _lib
    lib = _lib.load()

    class Event:
        def __init__(self, done):
            self.done = done

        def query(self):
            return self.done

    class Word:
        def __init__(self, value, done):
            self.event, self.value = Event(done), value

        def read(self):
            return [self.value]

    saved = list(_core._LATE_WORDS)
    try:
        _core._LATE_WORDS[:] = [Word(0, True), Word(16, False)]
        _core._check_late(lib)
        assert len(_core._LATE_WORDS) == 1
        _core._LATE_WORDS[0].event.done = True
        with pytest.raises(RuntimeError, match="bounded wait"):
            _core._check_late(lib)
        assert _core._LATE_WORDS == []
    finally:
        _core._LATE_WORDS[:] = saved
