"""rapidalign_b200.kde_gradients: the reference's float64 verification helpers
(kde_gradients.py:39-193) on the GPU, against fixtures produced by the
reference itself (tests/golden/make_golden.py: segmented_* carry the ragged
helper's outputs as raw_*, gradients_* the single-pair helpers with their
matrices).  Both sides are float64: agreement to 1e-10 relative."""
import numpy as np
import pytest
import torch

from conftest import golden_cases, load_golden

TOL = 1e-10


def rel(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    scale = max(float(np.max(np.abs(b))) if b.size else 0.0, 1e-300)
    return float(np.max(np.abs(a - b))) / scale if b.size else 0.0


def _np(t):
    return t.detach().cpu().numpy()


def test_cpu_tensors_are_refused():
    from rapidalign_b200 import kde_gradients as KG
    x = torch.zeros(3, 2, dtype=torch.float64)
    w = torch.ones(3, dtype=torch.float64)
    with pytest.raises(RuntimeError, match="CUDA"):
        KG.kde_mmd_backward_ragged(x, x, w, w, torch.tensor([0, 3]), torch.tensor([0, 3]), 0.5)


def test_float32_is_refused():
    from rapidalign_b200 import kde_gradients as KG
    x = torch.zeros(3, 2)
    w = torch.ones(3)
    with pytest.raises(ValueError, match="float64"):
        KG.kde_mmd_forward(x, x, w, w, 0.5)
    with pytest.raises(ValueError, match="float64"):
        KG.kde_mmd_backward_ragged(x, x, w, w, torch.tensor([0, 3]), torch.tensor([0, 3]), 0.5)


@pytest.mark.gpu
@pytest.mark.parametrize("name", golden_cases("segmented"))
def test_ragged_helper_matches_reference(name, cuda_device):
    from rapidalign_b200 import kde_gradients as KG
    z = load_golden(name)
    dev = cuda_device
    t = {k: torch.tensor(z[k], device=dev) for k in ("x", "y", "w_x", "w_y", "ptr_x", "ptr_y")}
    out = KG.kde_mmd_backward_ragged_cpu(t["x"], t["y"], t["w_x"], t["w_y"], t["ptr_x"],
                                         t["ptr_y"], float(z["sigma"]))
    for key, ref in (("Kxx", "raw_Kxx"), ("Kyy", "raw_Kyy"), ("Kxy", "raw_Kxy"),
                     ("x", "raw_gx"), ("y", "raw_gy"), ("w_x", "raw_gwx"), ("w_y", "raw_gwy"),
                     ("sigma_per_pair", "raw_gsigma_pairs")):
        assert rel(_np(out[key]), z[ref]) < TOL, key
    assert rel(_np(out["loss"]), z["raw_Kxx"] + z["raw_Kyy"] - 2 * z["raw_Kxy"]) < TOL
    assert abs(float(out["sigma_total"]) - float(z["raw_gsigma_pairs"].sum())) <= \
        TOL * max(1.0, float(np.abs(z["raw_gsigma_pairs"]).sum()))


@pytest.mark.gpu
@pytest.mark.parametrize("name", golden_cases("gradients"))
def test_single_pair_helpers_match_reference(name, cuda_device):
    from rapidalign_b200 import kde_gradients as KG
    z = load_golden(name)
    dev = cuda_device
    x, y, wx, wy = (torch.tensor(z[k], device=dev) for k in ("x", "y", "w_x", "w_y"))
    sigma = float(z["sigma"])
    out = KG.kde_mmd_backward_cpu(x, y, wx, wy, sigma)
    for key, ref in (("x", "grad_x"), ("y", "grad_y"), ("w_x", "grad_wx"), ("w_y", "grad_wy"),
                     ("sigma", "grad_sigma")):
        assert rel(_np(out[key]), z[ref]) < TOL, key
    fwd = out["forward"]
    assert isinstance(fwd, KG.KDEForwardResult)
    for key in ("loss", "Kxx", "Kyy", "Kxy", "Gxx", "Gyy", "Gxy", "diff_xx", "diff_yy",
                "diff_xy"):
        got = getattr(fwd, key)
        assert got.dtype == torch.float64 and got.is_cuda
        assert rel(_np(got), z[key]) < TOL, key


@pytest.mark.gpu
def test_ragged_helper_rejects_bad_ptr(cuda_device):
    from rapidalign_b200 import kde_gradients as KG
    dev = cuda_device
    x = torch.randn(5, 3, dtype=torch.float64, device=dev)
    w = torch.ones(5, dtype=torch.float64, device=dev)
    good = torch.tensor([0, 2, 5], device=dev)
    with pytest.raises(ValueError, match="ptr\\[-1\\] must equal"):
        KG.kde_mmd_backward_ragged(x, x, w, w, torch.tensor([0, 2, 4], device=dev), good, 0.5)
    with pytest.raises(ValueError, match="ptr offsets"):
        KG.kde_mmd_backward_ragged(x, x, w, w, torch.tensor([0, 3, 2, 5], device=dev),
                                   torch.tensor([0, 1, 2, 5], device=dev), 0.5)
    with pytest.raises(ValueError, match="same length"):
        KG.kde_mmd_backward_ragged(x, x, w, w, torch.tensor([0, 5], device=dev), good, 0.5)


@pytest.mark.gpu
def test_ragged_helper_agrees_with_fused_path(cuda_device):
    """The float64 helper and the fused float32 path (legacy segmented ops) on
    the same ragged batch, D=8: the fused path's stated tolerances."""
    from rapidalign_b200 import _cuda as C
    from rapidalign_b200 import kde_gradients as KG
    dev = cuda_device
    g = torch.Generator().manual_seed(5)
    ptr = torch.tensor([0, 40, 41, 130], device=dev)
    x = torch.randn(130, 8, generator=g, dtype=torch.float64).to(dev)
    y = (x + 0.1 * torch.randn(130, 8, generator=g, dtype=torch.float64).to(dev))
    wx = torch.rand(130, generator=g, dtype=torch.float64).to(dev) + 0.1
    wy = torch.rand(130, generator=g, dtype=torch.float64).to(dev) + 0.1
    ex = KG.kde_mmd_backward_ragged(x, y, wx, wy, ptr, ptr, 1.2)
    f = [t.float() for t in (x, y, wx, wy)]
    Kxx, Kyy, Kxy = C.kde_mmd_forward_segmented(*f, ptr, ptr, 1.2)
    for got, ref in ((Kxx, ex["Kxx"]), (Kyy, ex["Kyy"]), (Kxy, ex["Kxy"])):
        assert torch.allclose(got.double(), ref, rtol=2e-6, atol=0)
    gx, gy, gwx, gwy, gs = C.kde_mmd_backward_segmented(
        *f, ptr, ptr, torch.ones(3, dtype=torch.float64, device=dev), 1.2)
    for got, ref in ((gx, ex["x"]), (gy, ex["y"]), (gwx, ex["w_x"]), (gwy, ex["w_y"]),
                     (gs, ex["sigma_per_pair"])):
        assert float((got.double() - ref).abs().max()) <= 1e-4 * float(ref.abs().max())
