"""Rollout Routing Replay (R3) and the legacy router-logit record/replay.

R3 (reference ``lumenrl/moe/rollout_routing.py:71-152``): the rollout engine
returns, per row, the expert ids it selected for every token it ran through
the model (``[len, moe_layers, top_k]``, int16).  In training the packed
forward replays them: ``RoutingReplay.lookup(layer, T)`` hands the router the
ids for that layer in packed token order, and the router re-gathers the
weights from its LIVE softmax, so the router still gets gradients.  Lookup is
by layer index (activation recomputation replays layers in any order).
Tokens without a rollout decision (each row's last token, which the rollout
never fed back) carry -1 and keep the live top-k.

``R3Manager`` keeps the older trainer-internal replay (record the router
distribution during the old-log-prob pass, replay it in the update;
reference ``lumenrl/moe/r3_manager.py:20-77``).
"""

from __future__ import annotations

from typing import Optional

import torch
from torch import Tensor


def pack_rollout_routing(rows: list[Tensor], seq_lens: list[int], num_layers: int, top_k: int,
                         device) -> Tensor:
    """Concatenate per-row routes in packed token order, padding each row to
    its packed length with -1.  Returns [T, layers, k] int64."""
    parts = []
    for r, n in zip(rows, seq_lens):
        r = r.to(torch.long)
        if r.shape[0] >= n:
            parts.append(r[:n])
        else:
            pad = torch.full((n - r.shape[0], num_layers, top_k), -1, dtype=torch.long)
            parts.append(torch.cat([r, pad]))
    return torch.cat(parts).to(device)


class RoutingReplay:
    def __init__(self, packed: Tensor, moe_layers: list[int]) -> None:
        self.packed = packed                      # [T, L_moe, k]
        self.slot = {l: i for i, l in enumerate(moe_layers)}
        self.hits = 0
        self.tokens = 0

    @classmethod
    def from_rows(cls, rows: list[Tensor], seq_lens: list[int], args, device) -> "RoutingReplay":
        moe_layers = [i for i in range(args.num_layers) if args.is_moe_layer(i)]
        packed = pack_rollout_routing(rows, seq_lens, len(moe_layers), args.num_experts_per_tok, device)
        return cls(packed, moe_layers)

    def lookup(self, layer: int, num_tokens: int) -> Optional[Tensor]:
        if layer not in self.slot:
            return None
        ids = self.packed[:num_tokens, self.slot[layer]]
        self.tokens += ids.shape[0]
        self.hits += int((ids[:, 0] >= 0).sum())
        return ids

    def coverage(self) -> float:
        return self.hits / max(self.tokens, 1)


def apply_replay(probs: Tensor, live_ids: Tensor, replay_ids: Tensor) -> Tensor:
    """Rows with a full rollout decision take it; -1 rows keep ``live_ids``."""
    have = (replay_ids >= 0).all(-1, keepdim=True)
    return torch.where(have, replay_ids.clamp(min=0), live_ids)


class RouterRecorder:
    """Captures router distributions per layer (legacy logit replay)."""

    def __init__(self) -> None:
        self.store: dict[int, Tensor] = {}

    def record(self, layer: int, probs: Tensor) -> None:
        self.store[layer] = probs.detach().float().cpu()

    def clear(self) -> None:
        self.store.clear()


class R3Manager:
    """Trainer-internal replay: record during the old-log-prob forward,
    replay the recorded distribution in the policy update."""

    def __init__(self, enabled: bool = False, replay_mode: str = "distribution") -> None:
        self.enabled = enabled
        self.replay_mode = replay_mode
        self.recorder = RouterRecorder()
        self.replaying = False

    def start_record(self) -> None:
        self.replaying = False
        self.recorder.clear()

    def start_replay(self) -> None:
        self.replaying = True

    def stop(self) -> None:
        self.replaying = False

    def distribution(self, layer: int) -> Optional[Tensor]:
        return self.recorder.store.get(layer) if self.replaying else None

    def to_batch(self, batch) -> None:
        for layer, p in self.recorder.store.items():
            batch.add_router_distributions(layer, p)
