"""Learning-rate schedules (reference ``lumenrl/utils/lr_scheduler.py:20-82``
and the WSD schedule of ``lumenrl/trainer/bf16_optimizer.py``).

``lr_at(step)`` with warmup ``lr * (step+1)/warmup`` then constant / linear /
cosine (``num_cycles`` half-waves, floor ``min_lr_ratio``) / WSD
(warmup-stable-decay with the decay over the last ``wsd_decay_ratio``).
"""

from __future__ import annotations

import math


class LRSchedule:
    def __init__(self, base_lr: float, total_steps: int, warmup_steps: int = 0, style: str = "cosine",
                 min_lr_ratio: float = 0.0, num_cycles: float = 0.5, wsd_decay_ratio: float = 0.2,
                 wsd_decay_style: str = "cosine") -> None:
        self.base_lr = float(base_lr)
        self.total = max(int(total_steps), 1)
        self.warmup = max(int(warmup_steps), 0)
        self.style = style
        self.min_ratio = float(min_lr_ratio)
        self.num_cycles = float(num_cycles)
        self.wsd_decay_ratio = float(wsd_decay_ratio)
        self.wsd_decay_style = wsd_decay_style
        self.last_step = 0

    def _decay(self, progress: float, style: str) -> float:
        progress = min(max(progress, 0.0), 1.0)
        if style == "constant":
            return 1.0
        if style == "linear":
            f = 1.0 - progress
        else:
            f = max(0.0, 0.5 * (1.0 + math.cos(math.pi * 2.0 * self.num_cycles * progress)))
        return self.min_ratio + (1.0 - self.min_ratio) * f

    def lr_at(self, step: int) -> float:
        if self.warmup > 0 and step < self.warmup:
            return self.base_lr * float(step + 1) / float(self.warmup)
        if self.style == "constant":
            return self.base_lr
        if self.style.upper() == "WSD":
            decay_steps = max(int(self.total * self.wsd_decay_ratio), 1)
            start = self.total - decay_steps
            if step < start:
                return self.base_lr
            return self.base_lr * self._decay((step - start) / decay_steps, self.wsd_decay_style)
        span = max(self.total - self.warmup, 1)
        return self.base_lr * self._decay((step - self.warmup) / span, self.style)

    def step(self) -> float:
        self.last_step += 1
        return self.lr_at(self.last_step)

    @property
    def current(self) -> float:
        return self.lr_at(self.last_step)

    def state_dict(self) -> dict:
        return {"last_step": self.last_step}

    def load_state_dict(self, sd: dict) -> None:
        self.last_step = int(sd["last_step"])
