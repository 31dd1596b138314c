"""The oracle (oracle/kde_oracle.c + oracle/oracle.py) against golden vectors
produced by running the reference itself in float64 (tests/golden/make_golden.py).
This pins the oracle before any CUDA result is compared with it."""
import numpy as np
import pytest

from conftest import golden_cases, load_golden
from oracle import oracle as O

TOL = 1e-10  # both sides are float64; observed agreement ~1e-14


def rel(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    scale = max(float(np.max(np.abs(b))) if b.size else 0.0, 1e-300)
    return float(np.max(np.abs(a - b))) / scale if b.size else 0.0


# the loss fixtures (the learned-kernel module fixtures are checked in
# test_learned_kernel.py, the single-pair helper fixtures below)
LOSS_CASES = [n for n in golden_cases()
              if not n.startswith(("learned", "gradients", "pairwise"))]


@pytest.mark.parametrize("name", golden_cases("pairwise"))
def test_oracle_matches_pairwise_distance_loss(name):
    """algorithms.py:54-90: value and gradients (through sort and norm)."""
    z = load_golden(name)
    out, gs, gt = O.pairwise_distance_loss(z["src"], z["tgt"], z.get("src_batch"),
                                           z.get("tgt_batch"), str(z["reduction"]),
                                           upstream=z["upstream"])
    assert rel(out, z["out"]) < TOL
    assert rel(gs, z["grad_src"]) < TOL and rel(gt, z["grad_tgt"]) < TOL


@pytest.mark.parametrize("name", golden_cases("gradients"))
def test_oracle_matches_gradient_helpers(name):
    """kde_gradients.py single-pair helpers (raw weights, one pair)."""
    z = load_golden(name)
    n, m = z["x"].shape[0], z["y"].shape[0]
    px, py = np.array([0, n]), np.array([0, m])
    sigma = float(z["sigma"])
    Kxx, Kyy, Kxy = O.legacy_forward_segmented(z["x"], z["y"], z["w_x"], z["w_y"], px, py, sigma)
    assert rel(Kxx, np.atleast_1d(z["Kxx"])) < TOL and rel(Kyy, np.atleast_1d(z["Kyy"])) < TOL
    assert rel(Kxy, np.atleast_1d(z["Kxy"])) < TOL
    gx, gy, gwx, gwy, gs = O.legacy_backward_segmented(z["x"], z["y"], z["w_x"], z["w_y"], px, py,
                                                       np.ones(1), sigma)
    assert rel(gx, z["grad_x"]) < TOL and rel(gy, z["grad_y"]) < TOL
    assert rel(gwx, z["grad_wx"]) < TOL and rel(gwy, z["grad_wy"]) < TOL
    assert rel(gs, np.atleast_1d(z["grad_sigma"])) < TOL
    # the matrices by their definition (kde_gradients.py:32-36)
    d = z["x"][:, None, :] - z["y"][None, :, :]
    assert rel(d, z["diff_xy"]) < TOL
    assert rel(np.exp(-(d ** 2).sum(-1) / (2 * sigma ** 2)), z["Gxy"]) < TOL


@pytest.mark.parametrize("name", LOSS_CASES)
def test_oracle_matches_reference(name):
    z = load_golden(name)
    if name.startswith("segmented"):
        loss, g = O.segmented_kde_loss(z["x"], z["y"], z["w_x"], z["w_y"], z["ptr_x"],
                                       z["ptr_y"], float(z["sigma"]), z["upstream"])
        assert rel(loss, z["loss"]) < TOL
        for got, key in zip(g[:4], ["grad_x", "grad_y", "grad_wx", "grad_wy"]):
            assert rel(got, z[key]) < TOL, key
        assert rel(g[4], z["grad_sigma"]) < TOL
        # the legacy raw ops of the reference (kde_gradients ragged, D <= 3 here)
        Kxx, Kyy, Kxy = O.legacy_forward_segmented(z["x"], z["y"], z["w_x"], z["w_y"],
                                                   z["ptr_x"], z["ptr_y"], float(z["sigma"]))
        assert rel(Kxx, z["raw_Kxx"]) < TOL and rel(Kyy, z["raw_Kyy"]) < TOL
        assert rel(Kxy, z["raw_Kxy"]) < TOL
        P = z["ptr_x"].size - 1
        gx, gy, gwx, gwy, gs = O.legacy_backward_segmented(
            z["x"], z["y"], z["w_x"], z["w_y"], z["ptr_x"], z["ptr_y"], np.ones(P),
            float(z["sigma"]))
        assert rel(gx, z["raw_gx"]) < TOL and rel(gy, z["raw_gy"]) < TOL
        assert rel(gwx, z["raw_gwx"]) < TOL and rel(gwy, z["raw_gwy"]) < TOL
        assert rel(gs, z["raw_gsigma_pairs"]) < TOL
        return
    kw = dict(sigma=float(z["sigma"]), center=bool(z["center"]), cosine=bool(z["cosine"]),
              upstream=z["upstream"])
    if name.startswith("single"):
        r = O.kde_mmd_loss(z["x"], z["y"], z.get("x_w"), z.get("y_w"), **kw)
    elif name.startswith("pyg"):
        r = O.pyg_kde_mmd_loss(z["x"], z["y"], z["ptr_x"], z["ptr_y"], z.get("x_w"),
                               z.get("y_w"), **kw)
    else:
        r = O.kde_mmd_loss_dense(z["x"], z["y"], z["mask_x"], z["mask_y"], z.get("x_w"),
                                 z.get("y_w"), **kw)
    for key in ("loss", "Kxx", "Kyy", "Kxy"):
        assert rel(getattr(r, key), z[key]) < TOL, key
    assert rel(r.grad_x, z["grad_x"]) < TOL
    assert rel(r.grad_y, z["grad_y"]) < TOL
    if "grad_wx" in z:
        assert rel(r.grad_wx, z["grad_wx"]) < TOL
        assert rel(r.grad_wy, z["grad_wy"]) < TOL
    if "grad_sigma" in z:
        assert abs(r.grad_sigma - float(z["grad_sigma"])) <= TOL * max(abs(float(z["grad_sigma"])), 1e-300)
