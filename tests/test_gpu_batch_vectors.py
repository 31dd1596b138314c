"""Batch-vector inputs of ``pyg_kde_mmd_loss`` (rapidalign/kde.py:124-156).

The ptr offsets are built on the device (``ra_ptr_from_batch``) and checked
there: a call starts with the graph count of the previous batch-vector call
on the device, and a wrong count is found before any result is returned and
the call is repeated with the exact count.  These tests drive every branch --
first call, a repeated count, a changed count, empty graphs inside the batch,
and the reference's errors after a count has been remembered -- and compare
each result with the same batch given as ptr offsets.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _batch(rng, sizes, dev, dim=3):
    n = int(sum(sizes))
    x = torch.from_numpy(rng.standard_normal((n, dim)).astype(np.float32)).to(dev)
    b = torch.repeat_interleave(torch.arange(len(sizes)), torch.tensor(sizes)).to(dev)
    ptr = torch.tensor(np.concatenate([[0], np.cumsum(sizes)]), dtype=torch.long, device=dev)
    return x, b, ptr


def _same(a, b):
    for u, v in zip(a, b):
        assert torch.equal(u, v)


def test_changing_graph_counts_match_ptr_inputs(cuda_device):
    import rapidalign_b200 as ra
    dev = cuda_device
    rng = np.random.default_rng(3)
    for sizes in ([40, 7, 130], [40, 7, 130], [5, 6], [33, 1, 2, 90, 64], [33, 1, 2, 90, 64],
                  [2000]):
        x, bx, px = _batch(rng, sizes, dev)
        y, by, py = _batch(rng, [s + 3 for s in sizes], dev)
        got = ra.pyg_kde_mmd_loss(x, y, src_batch=bx, tgt_batch=by, sigma=0.3)
        ref = ra.pyg_kde_mmd_loss(x, y, src_ptr=px, tgt_ptr=py, sigma=0.3)
        assert got[0].shape == (len(sizes),)
        _same(got, ref)


def test_empty_graphs_inside_the_batch(cuda_device):
    """Graph ids that skip a value are empty graphs (bincount semantics)."""
    import rapidalign_b200 as ra
    dev = cuda_device
    rng = np.random.default_rng(4)
    x = torch.from_numpy(rng.standard_normal((9, 3)).astype(np.float32)).to(dev)
    y = torch.from_numpy(rng.standard_normal((7, 3)).astype(np.float32)).to(dev)
    bx = torch.tensor([0, 0, 0, 2, 2, 2, 2, 3, 3], device=dev)
    by = torch.tensor([0, 0, 2, 2, 3, 3, 3], device=dev)
    px = torch.tensor([0, 3, 3, 7, 9], device=dev)
    py = torch.tensor([0, 2, 2, 4, 7], device=dev)
    for _ in range(2):  # the second call starts from the remembered count
        got = ra.pyg_kde_mmd_loss(x, y, src_batch=bx, tgt_batch=by, sigma=0.4)
        ref = ra.pyg_kde_mmd_loss(x, y, src_ptr=px, tgt_ptr=py, sigma=0.4)
        _same(got, ref)


def test_reference_errors_after_a_remembered_count(cuda_device):
    import rapidalign_b200 as ra
    dev = cuda_device
    rng = np.random.default_rng(5)
    x, bx, _ = _batch(rng, [5, 5], dev)
    ra.pyg_kde_mmd_loss(x, x, src_batch=bx, tgt_batch=bx)  # remembers 2 graphs
    with pytest.raises(ValueError, match="sorted"):
        ra.pyg_kde_mmd_loss(x, x, src_batch=torch.tensor([0, 1] * 5, device=dev), tgt_batch=bx)
    with pytest.raises(ValueError, match="sorted"):
        ra.pyg_kde_mmd_loss(x, x, src_batch=bx, tgt_batch=torch.tensor([1, 0] * 5, device=dev))
    with pytest.raises(ValueError, match="non-negative"):
        ra.pyg_kde_mmd_loss(x, x, src_batch=bx - 1, tgt_batch=bx)
    with pytest.raises(ValueError, match="same length"):
        ra.pyg_kde_mmd_loss(x, x, src_batch=bx, tgt_batch=torch.zeros_like(bx))
    # and the next good call is right again
    x2, b2, p2 = _batch(rng, [3, 4, 5], dev)
    _same(ra.pyg_kde_mmd_loss(x2, x2, src_batch=b2, tgt_batch=b2),
          ra.pyg_kde_mmd_loss(x2, x2, src_ptr=p2, tgt_ptr=p2))


def test_gradients_through_the_batch_vector_path(cuda_device):
    import rapidalign_b200 as ra
    dev = cuda_device
    rng = np.random.default_rng(6)
    x, bx, px = _batch(rng, [100, 3, 700], dev)
    y, by, py = _batch(rng, [90, 8, 650], dev)
    grads = []
    for kw in (dict(src_batch=bx, tgt_batch=by), dict(src_batch=bx, tgt_batch=by),
               dict(src_ptr=px, tgt_ptr=py)):
        xs, ys = x.clone().requires_grad_(True), y.clone().requires_grad_(True)
        ra.pyg_kde_mmd_loss(xs, ys, sigma=0.25, **kw)[0].sum().backward()
        grads.append((xs.grad, ys.grad))
    # the default mode adds column sums atomically (order-dependent in the
    # last bits): equal within rounding, not bitwise
    for g in grads[:2]:
        for a, b in zip(g, grads[2]):
            assert float((a - b).abs().max()) <= 1e-6 * float(b.abs().max())


def test_ptr_from_batch_flags(cuda_device):
    """ra_ptr_from_batch through the C ABI: exact offsets and the flag bits."""
    from rapidalign_b200 import _lib
    lib = _lib.load()
    dev = cuda_device

    def run(batch, P):
        b = torch.tensor(batch, dtype=torch.long, device=dev)
        ptr = torch.full((P + 1,), -7, dtype=torch.long, device=dev)
        flags = torch.full((1,), -1, dtype=torch.int32, device=dev)
        rc = lib.ra_ptr_from_batch(b.data_ptr() if b.numel() else None, b.numel(), P,
                                   ptr.data_ptr(), flags.data_ptr(), _lib.stream_handle(dev))
        assert rc == 0
        return ptr.cpu().tolist(), int(flags.item())

    assert run([0, 0, 1, 3, 3], 4) == ([0, 2, 3, 3, 5], 0)
    assert run([], 3) == ([0, 0, 0, 0], 0)
    assert run([0, 0, 1], 4)[1] == _lib.RA_BATCH_COUNT
    assert run([0, 0, 1], 2) == ([0, 2, 3], 0)
    assert run([1, 0], 2)[1] & _lib.RA_BATCH_UNSORTED
    assert run([-1, 0], 1)[1] & _lib.RA_BATCH_NEGATIVE
