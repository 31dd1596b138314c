"""pairwise_distance_loss (algorithms.py:54-90) on the GPU against fixtures
produced by the reference (float64 autograd) and against the float64 oracle.
Distances are float32 on the GPU: losses within 1e-5 relative, gradients
within 1e-4 of their largest entry."""
import numpy as np
import pytest
import torch

from conftest import golden_cases, load_golden
from oracle import oracle as O

LOSS_REL = 1e-5


def _close(got, ref, rel):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    scale = np.maximum(np.abs(ref), 1e-30)
    assert np.all(np.abs(got - ref) <= rel * scale), float(np.max(np.abs(got - ref) / scale))


def _grad_close(got, ref):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    scale = max(float(np.max(np.abs(ref))), 1e-30)
    assert float(np.max(np.abs(got - ref))) <= 1e-4 * scale


def test_cpu_tensors_are_refused():
    import rapidalign_b200 as ra
    with pytest.raises(RuntimeError, match="CUDA"):
        ra.pairwise_distance_loss(torch.zeros(3, 2), torch.zeros(3, 2))


@pytest.mark.gpu
@pytest.mark.parametrize("name", golden_cases("pairwise"))
def test_pairwise_matches_reference(name, cuda_device):
    import rapidalign_b200 as ra
    z = load_golden(name)
    dev = cuda_device
    src = torch.tensor(z["src"], dtype=torch.float32, device=dev, requires_grad=True)
    tgt = torch.tensor(z["tgt"], dtype=torch.float32, device=dev, requires_grad=True)
    kw = {}
    if "src_batch" in z:
        kw = dict(src_batch=torch.tensor(z["src_batch"], device=dev),
                  tgt_batch=torch.tensor(z["tgt_batch"], device=dev))
    out = ra.pairwise_distance_loss(src, tgt, reduction=str(z["reduction"]), **kw)
    assert out.dtype == torch.float32 and out.shape == z["out"].shape
    _close(out.detach().double().cpu().numpy(), z["out"], LOSS_REL)
    (out.double() * torch.as_tensor(z["upstream"], device=dev)).sum().backward()
    _grad_close(src.grad.double().cpu().numpy(), z["grad_src"])
    _grad_close(tgt.grad.double().cpu().numpy(), z["grad_tgt"])


@pytest.mark.gpu
def test_pairwise_ragged_batch_matches_oracle(cuda_device):
    """Graphs of 0 (absent id), 1, 2 and up to 700 points, unsorted ids."""
    import rapidalign_b200 as ra
    rng = np.random.default_rng(90)
    sizes_s = [1, 2, 700, 64, 33]
    sizes_t = [3, 1, 650, 70, 33]
    src = rng.standard_normal((sum(sizes_s), 3)).astype(np.float32)
    tgt = (1.1 * rng.standard_normal((sum(sizes_t), 3))).astype(np.float32)
    ids = np.array([0, 2, 3, 5, 9])  # sorted unique ids with gaps
    bs = rng.permutation(np.repeat(ids, sizes_s))
    bt = rng.permutation(np.repeat(ids, sizes_t))
    dev = cuda_device
    st = torch.tensor(src, device=dev, requires_grad=True)
    tt = torch.tensor(tgt, device=dev, requires_grad=True)
    out = ra.pairwise_distance_loss(st, tt, torch.tensor(bs, device=dev),
                                    torch.tensor(bt, device=dev), reduction="none")
    up = rng.uniform(0.5, 1.5, len(ids))
    (out.double() * torch.as_tensor(up, device=dev)).sum().backward()
    ref, gs, gt = O.pairwise_distance_loss(src, tgt, bs, bt, "none", upstream=up)
    _close(out.detach().double().cpu().numpy(), ref, LOSS_REL)
    _grad_close(st.grad.double().cpu().numpy(), gs)
    _grad_close(tt.grad.double().cpu().numpy(), gt)


@pytest.mark.gpu
def test_pairwise_errors(cuda_device):
    import rapidalign_b200 as ra
    dev = cuda_device
    x = torch.randn(6, 3, device=dev)
    b = torch.tensor([0, 0, 1, 1, 2, 2], device=dev)
    with pytest.raises(ValueError, match="batch counts must match"):
        ra.pairwise_distance_loss(x, x, b, torch.zeros(6, dtype=torch.long, device=dev))
    with pytest.raises(ValueError, match="same length"):
        ra.pairwise_distance_loss(x, x, b[:5], b)
    with pytest.raises(ValueError, match="Unsupported reduction"):
        ra.pairwise_distance_loss(x, x, reduction="max")
    with pytest.raises(ValueError, match="shape"):
        ra.pairwise_distance_loss(x[0], x)
    # two graphs of one point each: 0 / 0
    one = ra.pairwise_distance_loss(x[:1], x[:1], reduction="none")
    assert torch.isnan(one).all()
