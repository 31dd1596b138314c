"""Generate the golden fixtures in ``tests/golden/*.npz`` from the reference.

Run with a checkout of the reference on the import path, e.g.::

    PYTHONPATH=<checkout of the reference> python tests/golden/make_golden.py

Every case runs the reference's own CPU code path in float64 with PyTorch
autograd (``rapidalign.kde``: kde.py:39-109, 211-299, 302-428;
``rapidalign.autograd_kde``: autograd_kde.py:16-129 CPU branch;
``rapidalign.kde_gradients``: kde_gradients.py:135-193) and stores inputs,
outputs and gradients.  Inputs are drawn in float32 and widened to float64, so
a float32 implementation sees bit-identical inputs.  The fixtures travel with
the repository; the reference does not.
"""
from __future__ import annotations

import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def f32(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.float32).to(torch.float64)


def grads_of(tensors, outputs, upstream):
    total = sum((u * o).sum() for u, o in zip(upstream, outputs) if u is not None)
    req = [t for t in tensors if t is not None and t.requires_grad]
    gs = torch.autograd.grad(total, req, allow_unused=True)
    it = iter(gs)
    out = []
    for t in tensors:
        if t is not None and t.requires_grad:
            g = next(it)
            out.append(None if g is None else g.detach().numpy())
        else:
            out.append(None)
    return out


def save(name, **arrays):
    clean = {k: np.asarray(v) for k, v in arrays.items() if v is not None}
    np.savez_compressed(os.path.join(HERE, name + ".npz"), **clean)
    print("wrote", name, sorted(clean))


def case_single(name, n, m, d, sigma, center, cosine, weights, sigma_grad, seed, upstream_kind):
    from rapidalign import kde_mmd_loss
    g = torch.Generator().manual_seed(seed)
    x = f32(torch.randn(n, d, generator=g))
    y = f32(x[:m] + 0.05 * torch.randn(m, d, generator=g)) if m <= n else \
        f32(torch.randn(m, d, generator=g))
    xw = f32(torch.rand(n, generator=g) + 0.1) if weights else None
    yw = f32(torch.rand(m, generator=g) + 0.1) if weights else None
    x.requires_grad_(True)
    y.requires_grad_(True)
    if xw is not None:
        xw.requires_grad_(True)
        yw.requires_grad_(True)
    sig = torch.tensor(sigma, dtype=torch.float64, requires_grad=True) if sigma_grad else sigma
    outs = kde_mmd_loss(x, y, xw, yw, sigma=sig, center=center, cosine=cosine)
    if upstream_kind == "loss":
        up = [1.0, 0.0, 0.0, 0.0]
    else:
        up = [1.0, 0.3, -0.5, 0.7]
    ups = [torch.tensor(u, dtype=torch.float64) for u in up]
    grads = grads_of([x, y, xw, yw, sig if sigma_grad else None], outs, ups)
    save(name, x=x.detach().numpy(), y=y.detach().numpy(),
         x_w=None if xw is None else xw.detach().numpy(),
         y_w=None if yw is None else yw.detach().numpy(),
         sigma=np.float64(sigma), center=np.bool_(center), cosine=np.bool_(cosine),
         sigma_grad=np.bool_(sigma_grad), upstream=np.array(up),
         loss=outs[0].detach().numpy(), Kxx=outs[1].detach().numpy(),
         Kyy=outs[2].detach().numpy(), Kxy=outs[3].detach().numpy(),
         grad_x=grads[0], grad_y=grads[1], grad_wx=grads[2], grad_wy=grads[3],
         grad_sigma=grads[4])


def case_pyg(name, sizes_x, sizes_y, d, sigma, center, cosine, weights, use_batch, seed):
    from rapidalign import pyg_kde_mmd_loss
    g = torch.Generator().manual_seed(seed)
    ptr_x = torch.tensor([0] + list(np.cumsum(sizes_x)), dtype=torch.long)
    ptr_y = torch.tensor([0] + list(np.cumsum(sizes_y)), dtype=torch.long)
    x = f32(torch.randn(int(ptr_x[-1]), d, generator=g))
    y = f32(torch.randn(int(ptr_y[-1]), d, generator=g))
    # targets: perturbed copies where sizes allow, to keep the loss small like real use
    for p in range(len(sizes_x)):
        k = min(sizes_x[p], sizes_y[p])
        y[ptr_y[p]:ptr_y[p] + k] = f32(x[ptr_x[p]:ptr_x[p] + k]
                                       + 0.05 * torch.randn(k, d, generator=g))
    xw = f32(torch.rand(x.shape[0], generator=g) + 0.1) if weights else None
    yw = f32(torch.rand(y.shape[0], generator=g) + 0.1) if weights else None
    x.requires_grad_(True)
    y.requires_grad_(True)
    if weights:
        xw.requires_grad_(True)
        yw.requires_grad_(True)
    kw = dict(sigma=sigma, center=center, cosine=cosine, src_w=xw, tgt_w=yw)
    if use_batch:
        bx = torch.repeat_interleave(torch.arange(len(sizes_x)), torch.tensor(sizes_x))
        by = torch.repeat_interleave(torch.arange(len(sizes_y)), torch.tensor(sizes_y))
        outs = pyg_kde_mmd_loss(x, y, src_batch=bx, tgt_batch=by, **kw)
    else:
        outs = pyg_kde_mmd_loss(x, y, src_ptr=ptr_x, tgt_ptr=ptr_y, **kw)
    P = len(sizes_x)
    up = np.stack([np.linspace(1.0, 2.0, P), np.linspace(0.2, -0.3, P),
                   np.linspace(-0.1, 0.4, P), np.linspace(0.5, 0.0, P)])
    ups = [torch.tensor(u) for u in up]
    grads = grads_of([x, y, xw, yw], outs, ups)
    save(name, x=x.detach().numpy(), y=y.detach().numpy(), ptr_x=ptr_x.numpy(),
         ptr_y=ptr_y.numpy(), x_w=None if xw is None else xw.detach().numpy(),
         y_w=None if yw is None else yw.detach().numpy(), sigma=np.float64(sigma),
         center=np.bool_(center), cosine=np.bool_(cosine), use_batch=np.bool_(use_batch),
         upstream=up, loss=outs[0].detach().numpy(), Kxx=outs[1].detach().numpy(),
         Kyy=outs[2].detach().numpy(), Kxy=outs[3].detach().numpy(),
         grad_x=grads[0], grad_y=grads[1], grad_wx=grads[2], grad_wy=grads[3])


def case_dense(name, lens_x, lens_y, nmax_x, nmax_y, d, sigma, center, cosine, weights,
               scramble, seed):
    from rapidalign import kde_mmd_loss_dense
    g = torch.Generator().manual_seed(seed)
    B = len(lens_x)
    x = f32(torch.randn(B, nmax_x, d, generator=g))
    y = f32(torch.randn(B, nmax_y, d, generator=g))
    k = min(nmax_x, nmax_y)
    y[:, :k] = f32(x[:, :k] + 0.05 * torch.randn(B, k, d, generator=g))
    mx = torch.zeros(B, nmax_x, dtype=torch.bool)
    my = torch.zeros(B, nmax_y, dtype=torch.bool)
    for b in range(B):
        if scramble:
            mx[b, torch.randperm(nmax_x, generator=g)[:lens_x[b]]] = True
            my[b, torch.randperm(nmax_y, generator=g)[:lens_y[b]]] = True
        else:
            mx[b, :lens_x[b]] = True
            my[b, :lens_y[b]] = True
    xw = f32(torch.rand(B, nmax_x, generator=g) + 0.1) if weights else None
    yw = f32(torch.rand(B, nmax_y, generator=g) + 0.1) if weights else None
    x.requires_grad_(True)
    y.requires_grad_(True)
    if weights:
        xw.requires_grad_(True)
        yw.requires_grad_(True)
    outs = kde_mmd_loss_dense(x, y, mx, my, x_w=xw, y_w=yw, sigma=sigma, center=center,
                              cosine=cosine)
    up = np.stack([np.linspace(1.0, 2.0, B), np.linspace(0.2, -0.3, B),
                   np.linspace(-0.1, 0.4, B), np.linspace(0.5, 0.0, B)])
    grads = grads_of([x, y, xw, yw], outs, [torch.tensor(u) for u in up])
    save(name, x=x.detach().numpy(), y=y.detach().numpy(), mask_x=mx.numpy(),
         mask_y=my.numpy(), x_w=None if xw is None else xw.detach().numpy(),
         y_w=None if yw is None else yw.detach().numpy(), sigma=np.float64(sigma),
         center=np.bool_(center), cosine=np.bool_(cosine), upstream=up,
         loss=outs[0].detach().numpy(), Kxx=outs[1].detach().numpy(),
         Kyy=outs[2].detach().numpy(), Kxy=outs[3].detach().numpy(),
         grad_x=grads[0], grad_y=grads[1], grad_wx=grads[2], grad_wy=grads[3])


def case_segmented(name, ptr_x, ptr_y, d, sigma, seed):
    """autograd_kde CPU branch + kde_gradients ragged (raw weights, may be negative)."""
    from rapidalign.autograd_kde import segmented_kde_loss
    from rapidalign.kde_gradients import kde_mmd_backward_ragged_cpu
    g = torch.Generator().manual_seed(seed)
    px = torch.tensor(ptr_x, dtype=torch.long)
    py = torch.tensor(ptr_y, dtype=torch.long)
    x = f32(torch.randn(int(px[-1]), d, generator=g)).requires_grad_(True)
    y = f32(torch.randn(int(py[-1]), d, generator=g)).requires_grad_(True)
    wx = f32(torch.randn(int(px[-1]), generator=g)).requires_grad_(True)
    wy = f32(torch.randn(int(py[-1]), generator=g)).requires_grad_(True)
    sig = torch.tensor(sigma, dtype=torch.float64, requires_grad=True)
    losses = segmented_kde_loss(x, y, wx, wy, px, py, sig)
    P = px.numel() - 1
    up = torch.linspace(0.5, 1.5, P, dtype=torch.float64)
    (losses * up).sum().backward()
    raw = kde_mmd_backward_ragged_cpu(x.detach(), y.detach(), wx.detach(), wy.detach(), px, py,
                                      sigma)
    save(name, x=x.detach().numpy(), y=y.detach().numpy(), w_x=wx.detach().numpy(),
         w_y=wy.detach().numpy(), ptr_x=px.numpy(), ptr_y=py.numpy(), sigma=np.float64(sigma),
         upstream=up.numpy(), loss=losses.detach().numpy(), grad_x=x.grad.numpy(),
         grad_y=y.grad.numpy(), grad_wx=wx.grad.numpy(), grad_wy=wy.grad.numpy(),
         grad_sigma=sig.grad.numpy(), raw_Kxx=raw["Kxx"].numpy(), raw_Kyy=raw["Kyy"].numpy(),
         raw_Kxy=raw["Kxy"].numpy(), raw_gx=raw["x"].numpy(), raw_gy=raw["y"].numpy(),
         raw_gwx=raw["w_x"].numpy(), raw_gwy=raw["w_y"].numpy(),
         raw_gsigma_pairs=raw["sigma_per_pair"].numpy())


def case_gradients(name, n, m, d, sigma, seed):
    """kde_gradients.py single-pair helpers: forward matrices and backward."""
    from rapidalign.kde_gradients import kde_mmd_backward_cpu
    g = torch.Generator().manual_seed(seed)
    x = f32(torch.randn(n, d, generator=g))
    y = f32(torch.randn(m, d, generator=g) * 1.1 + 0.1)
    wx = f32(torch.rand(n, generator=g) + 0.1)
    wy = f32(torch.rand(m, generator=g) + 0.1)
    out = kde_mmd_backward_cpu(x, y, wx, wy, sigma)
    fwd = out["forward"]
    save(name, x=x.numpy(), y=y.numpy(), w_x=wx.numpy(), w_y=wy.numpy(), sigma=np.float64(sigma),
         loss=fwd.loss.numpy(), Kxx=fwd.Kxx.numpy(), Kyy=fwd.Kyy.numpy(), Kxy=fwd.Kxy.numpy(),
         Gxx=fwd.Gxx.numpy(), Gyy=fwd.Gyy.numpy(), Gxy=fwd.Gxy.numpy(),
         diff_xx=fwd.diff_xx.numpy(), diff_yy=fwd.diff_yy.numpy(), diff_xy=fwd.diff_xy.numpy(),
         grad_x=out["x"].numpy(), grad_y=out["y"].numpy(), grad_wx=out["w_x"].numpy(),
         grad_wy=out["w_y"].numpy(), grad_sigma=out["sigma"].numpy())


def case_pairwise(name, sizes_src, sizes_tgt, d, reduction, shuffle, seed, no_batch=False):
    """algorithms.py:54-90 (float64, autograd through sort and norm); batch ids
    may be unsorted (the reference groups by value, not by position)."""
    from rapidalign.algorithms import pairwise_distance_loss
    g = torch.Generator().manual_seed(seed)
    src = f32(torch.randn(sum(sizes_src), d, generator=g)).requires_grad_(True)
    tgt = f32(1.05 * torch.randn(sum(sizes_tgt), d, generator=g)).requires_grad_(True)
    bs = torch.repeat_interleave(torch.arange(len(sizes_src)), torch.tensor(sizes_src))
    bt = torch.repeat_interleave(torch.arange(len(sizes_tgt)), torch.tensor(sizes_tgt))
    if shuffle:
        bs = bs[torch.randperm(bs.numel(), generator=g)]
        bt = bt[torch.randperm(bt.numel(), generator=g)]
    if no_batch:
        out = pairwise_distance_loss(src, tgt, reduction=reduction)
    else:
        out = pairwise_distance_loss(src, tgt, bs, bt, reduction=reduction)
    up = torch.linspace(0.5, 1.5, out.numel(), dtype=torch.float64).reshape(out.shape)
    (out * up).sum().backward()
    arrays = dict(src=src.detach().numpy(), tgt=tgt.detach().numpy(), out=out.detach().numpy(),
                  upstream=up.numpy(), grad_src=src.grad.numpy(), grad_tgt=tgt.grad.numpy(),
                  reduction=np.array(reduction))
    if not no_batch:
        arrays.update(src_batch=bs.numpy(), tgt_batch=bt.numpy())
    save(name, **arrays)


def case_learned(name, kind, n, m, seed):
    """learned_kernel.py modules (float64; the gate's float32 cast is undone by
    a forward pre-hook so that the whole module runs in float64)."""
    from rapidalign.learned_kernel import LearnedKernel, SingleSigmaKernel, StructuredKernel
    torch.manual_seed(seed)
    g = torch.Generator().manual_seed(seed + 1)
    x = f32(torch.randn(n, 2, generator=g))
    y = f32(1.1 * torch.randn(m, 2, generator=g) + 0.05)
    x.requires_grad_(True)
    y.requires_grad_(True)
    extra = {}
    if kind == "multi":
        mod = LearnedKernel(sigmas=(0.15, 0.3, 0.6), coord_dim=2).double()
        mod.gate.register_forward_pre_hook(lambda mdl, inp: (inp[0].double(),))
        loss = mod(x, y)
    elif kind == "single":
        mod = SingleSigmaKernel(init_sigma=0.3, use_weight_net=True, coord_dim=2).double()
        loss = mod(x, y)
    else:
        mod = StructuredKernel(init_sigma=0.3, feature_dim=5, descriptor_dim=4).double()
        fb = f32(torch.randn(n, 5, generator=g))
        ft = f32(torch.randn(m, 5, generator=g))
        db = f32(torch.randn(4, generator=g))
        dt = f32(torch.randn(4, generator=g))
        loss = mod(dict(pos=x, feat=fb, desc=db), dict(pos=y, feat=ft, desc=dt))
        extra = dict(feat_x=fb.numpy(), feat_y=ft.numpy(), desc_x=db.numpy(), desc_y=dt.numpy())
    loss.backward()
    params = {"p_" + k: v.detach().numpy() for k, v in mod.state_dict().items()}
    grads = {"g_" + k: prm.grad.numpy() for k, prm in mod.named_parameters()
             if prm.grad is not None}
    save(name, loss=loss.detach().numpy(), x=x.detach().numpy(), y=y.detach().numpy(),
         grad_x=x.grad.numpy(), grad_y=y.grad.numpy(), **extra, **params, **grads)


def main():
    torch.set_default_dtype(torch.float64)
    # single pair: the CPU-runnable headline shape (128 x 3, sigma 0.2, centred) and variants
    case_single("single_cfg1", 128, 128, 3, 0.2, True, False, False, False, 0, "loss")
    case_single("single_uncentred_allout", 96, 96, 3, 0.25, False, False, False, False, 1, "all")
    case_single("single_cosine_w", 64, 50, 3, 0.3, True, True, True, False, 2, "all")
    case_single("single_sigma_grad_w", 80, 64, 3, 0.2, True, False, True, True, 3, "all")
    case_single("single_d2", 40, 33, 2, 0.25, True, False, True, True, 4, "all")
    case_single("single_tiny", 1, 2, 3, 0.5, True, False, False, False, 5, "all")
    # ragged batches (ptr and batch-vector inputs, an empty graph on one side)
    case_pyg("pyg_uniform", [17, 1, 40, 2, 64, 33], [20, 3, 38, 2, 70, 31], 3, 0.25, True,
             False, False, False, 10)
    case_pyg("pyg_weighted_cosine", [30, 5, 70], [25, 9, 66], 3, 0.3, True, True, True, True, 11)
    case_pyg("pyg_uncentred_batch", [12, 0, 45, 7], [10, 6, 40, 9], 3, 0.2, False, False, False,
             True, 12)
    case_pyg("pyg_d2_weighted", [9, 23, 4], [11, 20, 6], 2, 0.4, True, False, True, False, 13)
    # dense padded batches: prefix masks (to_dense_batch layout) and scattered masks
    case_dense("dense_prefix", [12, 7, 10], [11, 10, 4], 12, 11, 3, 0.25, True, False, False,
               False, 20)
    case_dense("dense_scattered_w", [5, 9, 3], [6, 8, 8], 10, 9, 3, 0.3, True, False, True,
               True, 21)
    case_dense("dense_cosine_uncentred", [8, 16], [16, 12], 16, 16, 3, 0.25, False, True, False,
               False, 22)
    # the differentiable segmented op (raw, possibly negative weights, no centering)
    case_segmented("segmented_ref_test", [0, 3, 7], [0, 2, 5], 3, 0.35, 42)
    case_segmented("segmented_ragged", [0, 10, 11, 40, 40, 57], [0, 8, 20, 41, 44, 60], 3, 0.25,
                   7)
    case_segmented("segmented_d2", [0, 2, 5], [0, 3, 4], 2, 0.25, 6)
    # the float64 verification helpers (kde_gradients.py:39-132), one pair
    case_gradients("gradients_d3", 23, 17, 3, 0.4, 40)
    case_gradients("gradients_d16", 12, 9, 16, 1.3, 41)
    # the pairwise-distance spectrum loss (algorithms.py:54-90)
    case_pairwise("pairwise_mean", [12, 1, 30, 7], [10, 3, 33, 7], 3, "mean", False, 50)
    case_pairwise("pairwise_none_shuffled", [9, 20, 2], [11, 18, 5], 3, "none", True, 51)
    case_pairwise("pairwise_sum_d2", [25, 6], [20, 6], 2, "sum", False, 52)
    case_pairwise("pairwise_single", [40], [37], 3, "mean", False, 53, no_batch=True)
    # learned-kernel callers (learned_kernel.py:41-202)
    case_learned("learned_multi", "multi", 60, 45, 30)
    case_learned("learned_single", "single", 50, 64, 31)
    case_learned("learned_structured", "structured", 40, 37, 32)


if __name__ == "__main__":
    sys.exit(main())
