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
