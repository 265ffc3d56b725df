"""BF16 parameters with an fp32 master copy (reference
``lumenrl/trainer/bf16_optimizer.py:26-239``), used for the draft model.

Per step: gradients are converted to fp32, non-finite entries zeroed, clipped
by the global norm (fp32), AdamW runs on the fp32 masters and the result is
copied back to the bf16 parameters; LR follows cosine or WSD with warmup.
On CUDA the update is the fused AdamW kernel (bf16 write included).
"""

from __future__ import annotations

import math
from typing import Iterable

import torch

from lumenrl_b200.engine.training.lr_scheduler import LRSchedule
from lumenrl_b200.ops import reference as ref


class BF16Optimizer:
    def __init__(self, params: Iterable[torch.nn.Parameter], lr: float = 1e-4, betas=(0.9, 0.95), eps: float = 1e-8,
                 weight_decay: float = 0.0, max_grad_norm: float = 1.0, total_steps: int = 1000,
                 warmup_steps: int = 0, style: str = "cosine", min_lr_ratio: float = 0.0) -> None:
        self.params = [p for p in params if p.requires_grad]
        self.master = [p.detach().float().clone() for p in self.params]
        self.m = [torch.zeros_like(x) for x in self.master]
        self.v = [torch.zeros_like(x) for x in self.master]
        self.betas, self.eps, self.wd, self.max_norm = betas, eps, weight_decay, max_grad_norm
        self.sched = LRSchedule(lr, total_steps, warmup_steps, style, min_lr_ratio)
        self.step_count = 0

    @torch.no_grad()
    def step(self) -> dict:
        grads = []
        for p in self.params:
            g = p.grad.float() if p.grad is not None else torch.zeros_like(p, dtype=torch.float32)
            grads.append(torch.nan_to_num(g, nan=0.0, posinf=0.0, neginf=0.0))
        norm = math.sqrt(sum(float((g.double() ** 2).sum()) for g in grads)) if grads else 0.0
        clip = min(1.0, self.max_norm / (norm + 1e-6)) if self.max_norm else 1.0
        self.step_count += 1
        lr = self.sched.current
        b1, b2 = self.betas
        for p, mp, m, v, g in zip(self.params, self.master, self.m, self.v, grads):
            if p.is_cuda and p.dtype == torch.bfloat16 and mp.numel() % 4 == 0:
                from lumenrl_b200.ops.ext import ext
                ext().adamw_step(mp.view(-1), g.contiguous().view(-1), m.view(-1), v.view(-1), p.data.view(-1), lr,
                                 b1, b2, self.eps, self.wd, self.step_count, clip)
            else:
                ref.adamw_reference(mp, g, m, v, lr, b1, b2, self.eps, self.wd, self.step_count, clip)
                p.data.copy_(mp.to(p.dtype))
            p.grad = None
        self.sched.step()
        return {"grad_norm": norm, "lr": lr}

    def zero_grad(self) -> None:
        for p in self.params:
            p.grad = None
