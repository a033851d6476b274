"""Upload of a training step's host inputs (target image, W2C) that overlaps
the device's earlier work.

Each upload copies the host tensors on a side stream into one of two device
staging slots, then (on the caller's current stream, after that copy) into
the step's static input buffers. The next step's upload therefore runs while
the current step's kernels execute; a slot is reused only after the copy out
of it has run.
"""
from __future__ import annotations

from typing import Sequence

import torch


class InputStager:
    def __init__(self, device: torch.device):
        self.device = device
        self.stream = None  # created at the first host upload
        self._slots: list = [None, None]
        self._ready: list = []
        self._free: list = []
        self._next = 0

    def upload(self, sources: Sequence[torch.Tensor], dests: Sequence[torch.Tensor]) -> None:
        """dests[i] <- sources[i] (host or device), ordered before the work
        enqueued next on the current stream."""
        main = torch.cuda.current_stream(self.device)
        if all(s.device.type != "cpu" for s in sources):
            for s, d in zip(sources, dests):
                if s.data_ptr() != d.data_ptr():
                    d.copy_(s, non_blocking=True)
            return
        if self.stream is None:
            self.stream = torch.cuda.Stream(self.device)
            self._ready = [torch.cuda.Event(), torch.cuda.Event()]
            self._free = [torch.cuda.Event(), torch.cuda.Event()]
        k = self._next
        self._next ^= 1
        slot = self._slots[k]
        if slot is None or any(a.shape != d.shape or a.dtype != d.dtype for a, d in zip(slot, dests)):
            slot = self._slots[k] = [torch.empty_like(d) for d in dests]
        self.stream.wait_event(self._free[k])  # the slot's last contents were copied out
        with torch.cuda.stream(self.stream):
            for s, a in zip(sources, slot):
                a.copy_(s, non_blocking=True)
            self._ready[k].record(self.stream)
        main.wait_event(self._ready[k])
        for a, d in zip(slot, dests):
            d.copy_(a)
        self._free[k].record(main)
