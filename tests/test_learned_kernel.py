"""Learned-kernel modules (rapidalign/learned_kernel.py) on the CUDA path,
against golden fixtures made by the reference modules in float64
(tests/golden/make_golden.py).  Parameters are loaded from the fixtures, so
the reference's own initialisation is reproduced exactly."""
import numpy as np
import pytest
import torch

from conftest import load_golden

CASES = {
    "learned_multi": ("LearnedKernel", dict(sigmas=(0.15, 0.3, 0.6), coord_dim=2)),
    "learned_single": ("SingleSigmaKernel", dict(init_sigma=0.3, use_weight_net=True,
                                                 coord_dim=2)),
    "learned_structured": ("StructuredKernel", dict(init_sigma=0.3, feature_dim=5,
                                                    descriptor_dim=4)),
}


def _module(name):
    from rapidalign_b200 import learned_kernel as lk
    cls, kw = CASES[name]
    return getattr(lk, cls)(**kw)


def _state(z):
    return {k[2:]: torch.as_tensor(v) for k, v in z.items() if k.startswith("p_")}


@pytest.mark.parametrize("name", sorted(CASES))
def test_parameters_match_the_reference_layout(name):
    """Same parameter names and shapes as the reference modules (CPU only)."""
    z = load_golden(name)
    mod = _module(name)
    ref = _state(z)
    ours = mod.state_dict()
    assert sorted(ours) == sorted(ref)
    for k in ours:
        assert tuple(ours[k].shape) == tuple(ref[k].shape), k
    mod.load_state_dict({k: v.float() for k, v in ref.items()})


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(CASES))
def test_learned_kernel_matches_reference(name, cuda_device):
    z = load_golden(name)
    dev = cuda_device
    mod = _module(name)
    mod.load_state_dict({k: v.float() for k, v in _state(z).items()})
    mod = mod.to(dev)
    x = torch.tensor(z["x"], dtype=torch.float32, device=dev, requires_grad=True)
    y = torch.tensor(z["y"], dtype=torch.float32, device=dev, requires_grad=True)
    if name == "learned_structured":
        t = lambda k: torch.tensor(z[k], dtype=torch.float32, device=dev)
        loss = mod(dict(pos=x, feat=t("feat_x"), desc=t("desc_x")),
                   dict(pos=y, feat=t("feat_y"), desc=t("desc_y")))
    else:
        loss = mod(x, y)
    loss.backward()
    ref = float(z["loss"])
    got = float(loss.detach())
    assert abs(got - ref) <= 1e-5 * abs(ref), (got, ref)
    for pname, prm in mod.named_parameters():
        g_ref = z["g_" + pname]
        g = prm.grad.double().cpu().numpy()
        scale = max(float(np.max(np.abs(g_ref))), 1e-12)
        assert float(np.max(np.abs(g - g_ref))) / scale <= 1e-4, pname
    for got, key in ((x.grad, "grad_x"), (y.grad, "grad_y")):
        g_ref = z[key]
        err = float(np.max(np.abs(got.double().cpu().numpy() - g_ref))) / float(np.max(np.abs(g_ref)))
        assert err <= 1e-4, key
