"""Phase timers: CUDA events on the current stream when on GPU (device
time, read once per step), wall clock on CPU."""

from __future__ import annotations

import time

import torch


class PhaseTimer:
    def __init__(self, device) -> None:
        self.cuda = torch.device(device).type == "cuda"
        self._open: dict[str, object] = {}
        self._done: dict[str, tuple] = {}

    def start(self, name: str) -> None:
        if self.cuda:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            self._open[name] = e
        else:
            self._open[name] = time.perf_counter()

    def stop(self, name: str) -> None:
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
