"""Host-to-device staging of input batches on a side stream.

A training or evaluation loop that feeds the loss from host memory pays the
host-to-device copy of every batch.  ``DevicePrefetcher`` issues the copy of
the next batch on its own CUDA stream while the current batch is being
computed, so the copy engine and the SMs work at the same time; the compute
stream waits for a batch's copy on the device (an event), never on the host.

    pf = DevicePrefetcher(device)
    pf.put(first_host_batch)            # dict of pinned CPU tensors
    for step in range(n):
        batch = pf.get()                # device tensors of the staged batch
        if step + 1 < n:
            pf.put(next_host_batch)     # starts copying while this step runs
        loss = pyg_kde_mmd_loss(batch["x"], batch["y"], ...)

``get(prepare=...)`` can derive per-batch tensors on the copy stream (for
example ptr offsets with ``rapidalign_b200.batch_ptrs``).

Pinned (page-locked) host tensors copy asynchronously; pageable ones make
the copy synchronous and gain nothing.  The device buffers are allocated on
the copy stream and handed to the compute stream with ``record_stream``, so
the caching allocator does not reuse them while the compute still reads them.
"""
from __future__ import annotations

from typing import Callable, Dict, Optional

import torch

Tensor = torch.Tensor


class DevicePrefetcher:
    """One-batch-ahead staging of dicts of host tensors onto ``device``."""

    def __init__(self, device, stream: Optional[torch.cuda.Stream] = None):
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise RuntimeError("DevicePrefetcher stages batches onto a CUDA device")
        self.copy_stream = stream if stream is not None else torch.cuda.Stream(self.device)
        self._staged: Optional[Dict[str, Tensor]] = None
        self._ready: Optional[torch.cuda.Event] = None
        self.copy_start: Optional[torch.cuda.Event] = None  # of the latest put (timing)
        self.copy_end: Optional[torch.cuda.Event] = None

    def put(self, host_batch: Dict[str, Tensor]) -> None:
        """Start copying ``host_batch`` to the device on the copy stream."""
        if self._staged is not None:
            raise RuntimeError("a batch is already staged: get() it first")
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(self.copy_stream):
            start.record(self.copy_stream)
            staged = {k: v.to(self.device, non_blocking=True) for k, v in host_batch.items()}
            end.record(self.copy_stream)
        self._staged, self._ready = staged, end
        self.copy_start, self.copy_end = start, end

    def get(self, prepare: Optional[Callable[[Dict[str, Tensor]], Dict[str, Tensor]]] = None
            ) -> Dict[str, Tensor]:
        """The staged batch, usable on the current stream (which waits for
        its copy on the device).

        ``prepare(batch)``, if given, runs first on the copy stream and its
        returned tensors join the batch: per-batch work that needs a host
        synchronisation, e.g. ptr offsets from batch vectors (``batch_ptrs``),
        then waits for the copy only -- issued a step earlier, it is done --
        instead of for the compute stream's queue."""
        if self._staged is None:
            raise RuntimeError("no batch staged: put() one first")
        if prepare is not None:
            with torch.cuda.stream(self.copy_stream):
                self._staged.update(prepare(self._staged))
                self._ready = torch.cuda.Event()
                self._ready.record(self.copy_stream)
        cur = torch.cuda.current_stream(self.device)
        cur.wait_event(self._ready)
        for t in self._staged.values():
            t.record_stream(cur)
        out, self._staged, self._ready = self._staged, None, None
        return out


__all__ = ["DevicePrefetcher"]
