"""ra_mmd_outputs / ra_mmd_outputs_backward: the loss and the three sums in
the caller's dtype in one launch, and dL/dK in one launch, against the tensor
expressions they replace (rapidalign/kde.py:103-107: Kxx + Kyy - 2 Kxy, or
1 - Kxy / sqrt(max(Kxx Kyy, eps)), then .to(dtype))."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _reference(K, cosine, eps, dtype):
    Kxx, Kyy, Kxy = K
    loss = (1.0 - Kxy / (Kxx * Kyy).clamp_min(eps).sqrt()) if cosine else Kxx + Kyy - 2.0 * Kxy
    return loss.to(dtype), Kxx.to(dtype), Kyy.to(dtype), Kxy.to(dtype)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64, torch.bfloat16])
@pytest.mark.parametrize("cosine", [False, True])
def test_outputs_and_gradients_match_the_tensor_expressions(dtype, cosine, cuda_device):
    from rapidalign_b200._core import mmd_outputs
    dev = cuda_device
    g = torch.Generator().manual_seed(7 + int(cosine))
    P = 37
    base = torch.rand(3 * P, generator=g, dtype=torch.float64) + 0.05
    base[:3] = 1e-6  # a product below eps: the clamp's zero-gradient branch
    eps = 1e-8
    ups = [torch.rand(P, generator=g, dtype=torch.float64).to(dev) for _ in range(4)]

    def run(fn):
        Kb = base.clone().to(dev).requires_grad_(True)
        K = (Kb[:P], Kb[P:2 * P], Kb[2 * P:])
        outs = fn(K)
        total = sum((u.to(o.dtype) * o).sum() for u, o in zip(ups, outs))
        total.backward()
        return [o.detach().double().cpu() for o in outs], Kb.grad.cpu()

    got, ggot = run(lambda K: mmd_outputs(*K, cosine, eps, dtype))
    ref, gref = run(lambda K: _reference(K, cosine, eps, dtype))
    for a, b in zip(got, ref):
        assert torch.equal(a, b)  # same float64 expressions, same rounding
    assert torch.allclose(ggot, gref, rtol=1e-12, atol=1e-14)
