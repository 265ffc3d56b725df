"""Step- and rank-gated profiling (reference ``lumenrl/utils/profiler.py:29-292``).

Backends (``profiler.tool``):
* ``torch``: ``torch.profiler`` with optional (skip_first, wait, warmup,
  active, repeat) schedule; one chrome trace per rank and step under
  ``save_path``;
* ``nvtx``: NVTX ranges only (``range(name)`` context), for an external
  Nsight Systems / Compute capture;
* ``ncu``: emits the ``ncu`` command line to capture one kernel of the
  configured steps (always with ``--clock-control none``).
Profiling is active only on the selected ranks (``all_ranks`` or ``ranks``,
default rank 0) and steps (``steps``; all when empty).
"""

from __future__ import annotations

import contextlib
import os
from typing import Optional

import torch


class DistProfiler:
    def __init__(self, cfg, rank: int = 0) -> None:
        self.cfg = cfg
        self.rank = rank
        ranks = list(cfg.ranks) if cfg.ranks else [0]
        self.enabled = bool(cfg.enable) and (cfg.all_ranks or rank in ranks)
        self.steps = set(cfg.steps or [])
        self._prof = None
        self._step = None

    def active_for(self, step: int) -> bool:
        return self.enabled and (not self.steps or step in self.steps)

    def start(self, step: int) -> None:
        self._step = step
        if not self.active_for(step) or self.cfg.tool != "torch":
            return
        tc = self.cfg.tool_config
        contents = getattr(tc, "contents", ["cpu", "cuda"]) if tc is not None else ["cpu", "cuda"]
        acts = [torch.profiler.ProfilerActivity.CPU]
        if "cuda" in contents and torch.cuda.is_available():
            acts.append(torch.profiler.ProfilerActivity.CUDA)
        sched = None
        sc = getattr(tc, "schedule", None)
        if sc is not None and getattr(sc, "active", 0) > 0:
            sched = torch.profiler.schedule(skip_first=sc.skip_first, wait=sc.wait, warmup=sc.warmup,
                                            active=sc.active, repeat=sc.repeat)
        self._prof = torch.profiler.profile(activities=acts, schedule=sched, record_shapes="shapes" in contents,
                                            profile_memory="memory" in contents, with_stack="stack" in contents)
        self._prof.__enter__()

    def mark(self) -> None:
        if self._prof is not None:
            self._prof.step()

    def stop(self) -> Optional[str]:
        if self._prof is None:
            return None
        self._prof.__exit__(None, None, None)
        os.makedirs(self.cfg.save_path, exist_ok=True)
        path = os.path.join(self.cfg.save_path, f"trace_rank{self.rank}_step{self._step}.json")
        self._prof.export_chrome_trace(path)
        self._prof = None
        return path

    @contextlib.contextmanager
    def range(self, name: str):
        if self.enabled and torch.cuda.is_available():
            torch.cuda.nvtx.range_push(name)
            try:
                yield
            finally:
                torch.cuda.nvtx.range_pop()
        else:
            yield

    def ncu_command(self, kernel_regex: str, cmd: str, launches: int = 3, skip: int = 0) -> str:
        return (f"ncu --set full --clock-control none -k regex:{kernel_regex} -s {skip} -c {launches} "
                f"-o {os.path.join(self.cfg.save_path, 'prof')} {cmd}")
