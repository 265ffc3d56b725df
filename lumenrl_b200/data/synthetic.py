"""Synthetic prompt sources (uniform random token ids by seed).

``SyntheticPrompts(num_prompts_per_step, prompt_len, low, high, seed)`` yields
the same prompts for the same (seed, step, rank) on every run, so runs and
ranks are reproducible without a dataset.
"""

from __future__ import annotations

import torch


class SyntheticPrompts:
    def __init__(self, prompt_len: int, low: int, high: int, seed: int = 0) -> None:
        self.prompt_len, self.low, self.high, self.seed = prompt_len, low, high, seed
        self.cursor = 0

    def batch(self, n: int, step: int, rank: int = 0) -> list[list[int]]:
        g = torch.Generator().manual_seed(self.seed * 1_000_003 + step * 7919 + rank)
        ids = torch.randint(self.low, self.high, (n, self.prompt_len), generator=g)
        self.cursor = step + 1
        return ids.tolist()

    def batch_tensor(self, n: int, step: int, rank: int = 0, pin: bool = False, round: int = 0) -> torch.Tensor:
        """Same prompts as ``batch`` as an int64 [n, prompt_len] host tensor
        (page-locked when ``pin``, for an asynchronous host->device copy).
        ``round`` > 0 draws fresh prompts for the same step (DAPO refill)."""
        g = torch.Generator().manual_seed(self.seed * 1_000_003 + step * 7919 + rank + round * 104_729)
        ids = torch.randint(self.low, self.high, (n, self.prompt_len), generator=g)
        self.cursor = step + 1
        return ids.pin_memory() if pin else ids

    def state_dict(self) -> dict:
        return {"cursor": self.cursor, "seed": self.seed}

    def load_state_dict(self, sd: dict) -> None:
        self.cursor = int(sd["cursor"])
