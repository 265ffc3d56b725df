"""Phase timers: CUDA events on the current stream when on GPU (device
time, read once per step), wall clock on CPU."""

from __future__ import annotations

import time

import torch


class PhaseTimer:
    """``start(name)`` / ``stop(name)`` bracket a phase.  With ``nvtx`` (on
    GPU) every phase is also an NVTX range, so an external Nsight capture
    shows the step's phases on the timeline."""

    def __init__(self, device, nvtx: bool = False) -> None:
        self.cuda = torch.device(device).type == "cuda"
        self.nvtx = bool(nvtx) and self.cuda
        self._open: dict[str, object] = {}
        self._done: dict[str, tuple] = {}
        self._ranges: dict[str, int] = {}

    def start(self, name: str) -> None:
        if self.nvtx:
            self._ranges[name] = torch.cuda.nvtx.range_start(name)
        if self.cuda:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            self._open[name] = e
        else:
            self._open[name] = time.perf_counter()

    def stop(self, name: str) -> None:
        if self.nvtx and name in self._ranges:
            torch.cuda.nvtx.range_end(self._ranges.pop(name))
        s = self._open.pop(name)
        if self.cuda:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            self._done[name] = (s, e)
        else:
            self._done[name] = (s, time.perf_counter())

    def collect(self) -> dict[str, float]:
        out = {}
        if self.cuda:
            torch.cuda.synchronize()
            for k, (s, e) in self._done.items():
                out[k] = s.elapsed_time(e) / 1e3
        else:
            for k, (s, e) in self._done.items():
                out[k] = e - s
        self._done.clear()
        return out
