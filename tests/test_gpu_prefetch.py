"""rapidalign_b200.prefetch.DevicePrefetcher: staged batches arrive intact on
the device, the compute stream sees them complete, misuse raises."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_prefetched_batches_are_exact(cuda_device):
    from rapidalign_b200.prefetch import DevicePrefetcher
    pf = DevicePrefetcher(cuda_device)
    host = [{"x": torch.randn(100_000, 3).pin_memory(),
             "b": torch.arange(100_000, dtype=torch.long).pin_memory()} for _ in range(4)]
    pf.put(host[0])
    sums = []
    for i in range(4):
        batch = pf.get()
        if i + 1 < 4:
            pf.put(host[i + 1])
        # use the batch on the current stream right away
        sums.append((batch["x"].double().sum(), batch["b"].sum()))
    for (sx, sb), h in zip(sums, host):
        assert float(sx) == pytest.approx(float(h["x"].double().sum()), rel=1e-12)
        assert int(sb) == int(h["b"].sum())


def test_prefetcher_misuse_raises(cuda_device):
    from rapidalign_b200.prefetch import DevicePrefetcher
    pf = DevicePrefetcher(cuda_device)
    with pytest.raises(RuntimeError, match="no batch staged"):
        pf.get()
    pf.put({"x": torch.zeros(4).pin_memory()})
    with pytest.raises(RuntimeError, match="already staged"):
        pf.put({"x": torch.zeros(4).pin_memory()})


def test_prepare_runs_on_the_copy_stream(cuda_device):
    """get(prepare=batch_ptrs...) hands over ptr offsets with the batch; the
    loss through them equals the loss through the batch vectors."""
    import numpy as np
    import rapidalign_b200 as ra
    from rapidalign_b200.prefetch import DevicePrefetcher
    rng = np.random.default_rng(3)
    sizes = [40, 7, 90]
    host = {"x": torch.tensor(rng.standard_normal((sum(sizes), 3)), dtype=torch.float32),
            "b": torch.repeat_interleave(torch.arange(3), torch.tensor(sizes))}
    host["y"] = host["x"] + 0.05
    host = {k: v.pin_memory() for k, v in host.items()}

    def prepare(t):
        px, py = ra.batch_ptrs(t["b"], t["b"])
        return {"px": px, "py": py}

    pf = DevicePrefetcher(cuda_device)
    pf.put(host)
    t = pf.get(prepare=prepare)
    assert t["px"].tolist() == [0, 40, 47, 137]
    a = ra.pyg_kde_mmd_loss(t["x"], t["y"], src_ptr=t["px"], tgt_ptr=t["py"], sigma=0.3)
    b = ra.pyg_kde_mmd_loss(t["x"], t["y"], src_batch=t["b"], tgt_batch=t["b"], sigma=0.3)
    for u, v in zip(a, b):
        assert torch.equal(u, v)
