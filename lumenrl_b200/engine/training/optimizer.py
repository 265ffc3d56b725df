"""Sharded AdamW over the flat parameter buffer (ZeRO-style distributed
optimizer; reference: FSDP2 ``fully_shard`` + ``MixedPrecisionPolicy(param=bf16,
reduce=fp32)`` in ``lumenrl/engine/training/fsdp_backend.py:369-445`` and the
Megatron distributed optimizer).

Per rank: the full bf16 weights ``w16`` (resident: they are also the rollout
weights), the full fp32 gradient accumulator ``grad``, and an fp32 master /
Adam-m / Adam-v SHARD of ``numel / world`` elements.

``step``:
  1. reduce-scatter ``grad`` (SUM) into this rank's shard,
  2. global grad norm (sum of squares all-reduced), clip coefficient, skip the
     update if the norm is not finite (reference ``fsdp_engine.py:548-567``),
  3. AdamW on the shard; the new bf16 values are written straight into this
     rank's slice of ``w16`` (fused cast),
  4. all-gather the bf16 slices into every rank's ``w16`` -- this IS the
     trainer->rollout weight sync and the parameter all-gather of the next
     training step.
Steps 1 and 3-4 run as fused NVLink kernels on multi-GPU CUDA jobs
(``parallel.fused_comm``); NCCL / gloo collectives otherwise.
"""

from __future__ import annotations

import math
import time
from typing import Optional

import torch
import torch.distributed as dist
from torch import Tensor

from lumenrl_b200.ops import reference as ref


class ShardedFlatAdamW:
    def __init__(self, w16: Tensor, world: int = 1, rank: int = 0, lr: float = 1e-6, betas=(0.9, 0.999),
                 eps: float = 1e-8, weight_decay: float = 0.01, max_grad_norm: float = 1.0,
                 comm=None, grad_dtype: torch.dtype = torch.float32, group=None) -> None:
        n = w16.numel()
        if n % (world * 128):
            raise ValueError("flat buffer must be padded to a multiple of world * 128 elements")
        self.w16, self.world, self.rank = w16, world, rank
        self.shard = n // world
        self.lo, self.hi = rank * self.shard, (rank + 1) * self.shard
        dev = w16.device
        self.master = w16[self.lo: self.hi].float().clone()
        self.m = torch.zeros_like(self.master)
        self.v = torch.zeros_like(self.master)
        fused = comm is not None and hasattr(comm, "fused_step")
        self.grad = comm.grads.tensor if fused else torch.zeros(n, dtype=grad_dtype, device=dev)
        self.grad_shard = self.grad[self.lo: self.hi] if world == 1 else torch.zeros(self.shard, dtype=torch.float32,
                                                                                     device=dev)
        self.fused = fused
        self.lr, self.betas, self.eps, self.wd = lr, betas, eps, weight_decay
        self.max_grad_norm = max_grad_norm
        self.step_count = 0
        self.comm = comm
        self.group = group          # process group of the data-parallel replicas (None = world)
        self.last_timing: dict[str, float] = {}

    # -- collectives --------------------------------------------------------------
    def _reduce_scatter(self) -> None:
        if self.world == 1:
            return
        if self.comm is not None and hasattr(self.comm, "reduce_scatter_sum"):
            self.comm.reduce_scatter_sum(self.grad, self.grad_shard)
        elif self.grad.is_cuda:
            dist.reduce_scatter_tensor(self.grad_shard, self.grad, group=self.group)
        else:  # gloo has no reduce-scatter
            dist.all_reduce(self.grad, group=self.group)
            self.grad_shard.copy_(self.grad[self.lo: self.hi])

    def _all_gather(self) -> None:
        if self.world == 1:
            return
        if self.comm is not None and hasattr(self.comm, "all_gather"):
            self.comm.all_gather(self.w16, self.lo, self.hi)
        elif self.w16.is_cuda:
            dist.all_gather_into_tensor(self.w16, self.w16[self.lo: self.hi].clone(), group=self.group)
        else:
            parts = list(self.w16.view(self.world, -1).unbind(0))
            dist.all_gather(parts, self.w16[self.lo: self.hi].clone(), group=self.group)

    def _global_norm(self) -> float:
        g = self.grad_shard
        if g.is_cuda:
            from lumenrl_b200.ops.ext import ext
            sq = ext().sumsq(g)
        else:
            sq = (g.double() ** 2).sum().float().reshape(1)
        if self.world > 1:
            dist.all_reduce(sq, group=self.group)
        return float(sq.sqrt().item())

    # -- update -------------------------------------------------------------------
    @torch.no_grad()
    def step(self, lr: Optional[float] = None) -> dict[str, float]:
        lr = self.lr if lr is None else lr
        if self.fused:
            # one kernel pair over NVLink peer memory: reduce-scatter + norm, then
            # clip + AdamW + bf16 broadcast into every rank's resident weights
            norm, skipped = self.comm.fused_step(self.lo, self.shard, self.master, self.grad_shard, self.m, self.v,
                                                 lr, self.betas, self.eps, self.wd, self.step_count + 1,
                                                 self.max_grad_norm)
            if not skipped:
                self.step_count += 1
            self.grad.zero_()
            self.last_timing = dict(self.comm.last_timing)
            clip = min(1.0, self.max_grad_norm / (norm + 1e-6)) if self.max_grad_norm else 1.0
            return {"grad_norm": norm, "skipped": float(skipped), "lr": lr, "clip_coef": clip}
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)] if self.w16.is_cuda else None
        if ev:
            ev[0].record()
        t0 = time.perf_counter()
        self._reduce_scatter()
        norm = self._global_norm()
        if ev:
            ev[1].record()
        t1 = time.perf_counter()
        clip = 1.0
        if self.max_grad_norm and self.max_grad_norm > 0:
            clip = min(1.0, self.max_grad_norm / (norm + 1e-6))
        skipped = not math.isfinite(norm)
        if not skipped:
            self.step_count += 1
            b1, b2 = self.betas
            if self.master.is_cuda:
                from lumenrl_b200.ops.ext import ext
                ext().adamw_step(self.master, self.grad_shard, self.m, self.v, self.w16[self.lo: self.hi], lr, b1, b2,
                                 self.eps, self.wd, self.step_count, clip)
            else:
                ref.adamw_reference(self.master, self.grad_shard, self.m, self.v, lr, b1, b2, self.eps, self.wd,
                                    self.step_count, clip)
                self.w16[self.lo: self.hi].copy_(self.master.to(self.w16.dtype))
            self._all_gather()
        if ev:
            ev[2].record()
            ev[2].synchronize()
            # opt_rs_s: gradient reduce-scatter + global norm; opt_bcast_s: from
            # the reduced gradients to published bf16 weights (AdamW with the
            # cast fused into the resident buffer, then the all-gather)
            self.last_timing = {"opt_rs_s": ev[0].elapsed_time(ev[1]) / 1e3,
                                "opt_bcast_s": ev[1].elapsed_time(ev[2]) / 1e3}
        else:
            self.last_timing = {"opt_rs_s": t1 - t0, "opt_bcast_s": time.perf_counter() - t1}
        self.grad.zero_()
        if self.world > 1:
            self.grad_shard.zero_()
        return {"grad_norm": norm, "skipped": float(skipped), "lr": lr, "clip_coef": clip}

    def zero_grad(self) -> None:
        self.grad.zero_()

    # -- checkpoint -------------------------------------------------------------------
    def state_dict(self) -> dict:
        return {"master": self.master, "m": self.m, "v": self.v, "step": self.step_count,
                "world": self.world, "rank": self.rank}

    def load_state_dict(self, sd: dict) -> None:
        if sd["world"] != self.world:
            raise ValueError(f"optimizer shard was saved with world={sd['world']}, now {self.world}")
        self.master.copy_(sd["master"])
        self.m.copy_(sd["m"])
        self.v.copy_(sd["v"])
        self.step_count = int(sd["step"])
        self.w16[self.lo: self.hi].copy_(self.master.to(self.w16.dtype))
        self._all_gather()

    def offload(self) -> None:
        """Move master/m/v to pinned host memory (reference optimizer offload)."""
        for name in ("master", "m", "v"):
            t = getattr(self, name)
            if t.is_cuda:
                h = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
                h.copy_(t, non_blocking=True)
                setattr(self, name, h)
        torch.cuda.synchronize() if torch.cuda.is_available() else None

    def reload(self, device) -> None:
        for name in ("master", "m", "v"):
            t = getattr(self, name)
            if not t.is_cuda and torch.device(device).type == "cuda":
                setattr(self, name, t.to(device, non_blocking=True))
