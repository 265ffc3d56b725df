"""MoE router diagnostics and expert resharding (reference:
``lumenrl/moe/moe_utils.py:143-188``, ``lumenrl/moe/expert_parallel.py:18-132``).

- ``router_entropy`` / ``expert_utilization``: how peaked the router is and
  how evenly the routed assignments spread over the experts.
- ``RouterStats``: device-side accumulators filled by the MoE layers during a
  training step (no host read per layer or per micro-batch); ``summary()``
  reads them once and returns the step's metrics.
- ``reshard_experts``: re-partition stacked expert tensors ([E_local, ...]
  per expert-parallel rank) from a training EP width to an inference EP
  width, in either direction.
"""

from __future__ import annotations

from typing import Optional

import torch
from torch import Tensor


def router_entropy(probs: Tensor) -> Tensor:
    """Mean Shannon entropy (nats) of the per-token router distributions
    ``probs`` [T, E] (softmax outputs)."""
    p = probs.float().clamp_min(0)
    return -(p * torch.log(p.clamp_min(1e-30))).sum(-1).mean()


def expert_utilization(counts: Tensor) -> dict:
    """Statistics of routed-assignment counts per expert (``counts`` [E]):
    share of the busiest / idlest expert, max over mean (1 = perfectly even),
    coefficient of variation and the number of experts that got nothing."""
    c = counts.double()
    total = float(c.sum())
    E = c.numel()
    if total <= 0:
        return {"max_share": 0.0, "min_share": 0.0, "max_over_mean": 0.0, "cv": 0.0, "dead_experts": E}
    share = c / total
    mean = total / E
    return {"max_share": float(share.max()), "min_share": float(share.min()),
            "max_over_mean": float(c.max() / mean), "cv": float(c.std(unbiased=False) / mean),
            "dead_experts": int((c == 0).sum())}


class RouterStats:
    """Per-layer router statistics accumulated on the device over a step."""

    def __init__(self, num_layers: int, num_experts: int, device) -> None:
        self.entropy_sum = torch.zeros(num_layers, dtype=torch.float64, device=device)
        self.tokens = torch.zeros(num_layers, dtype=torch.float64, device=device)
        self.counts = torch.zeros(num_layers, num_experts, dtype=torch.float64, device=device)

    @torch.no_grad()
    def observe(self, layer: int, probs: Tensor, ids: Tensor) -> None:
        """``probs`` [T, E] router softmax, ``ids`` [T, k] chosen experts."""
        p = probs.float().clamp_min(0)
        self.entropy_sum[layer] += -(p * torch.log(p.clamp_min(1e-30))).sum().double()
        self.tokens[layer] += probs.shape[0]
        self.counts[layer].index_add_(0, ids.reshape(-1).long(),
                                      torch.ones(ids.numel(), dtype=torch.float64, device=ids.device))

    def reset(self) -> None:
        self.entropy_sum.zero_()
        self.tokens.zero_()
        self.counts.zero_()

    def summary(self, prefix: str = "moe/") -> dict:
        """One host read: mean router entropy and the utilisation statistics
        of the counts of the MoE layers that saw tokens."""
        ent, tok, cnt = (t.cpu() for t in (self.entropy_sum, self.tokens, self.counts))
        seen = tok > 0
        if not bool(seen.any()):
            return {}
        util = [expert_utilization(cnt[i]) for i in range(cnt.shape[0]) if bool(seen[i])]
        return {prefix + "router_entropy": float((ent[seen] / tok[seen]).mean()),
                prefix + "expert_max_over_mean": max(u["max_over_mean"] for u in util),
                prefix + "expert_cv": sum(u["cv"] for u in util) / len(util),
                prefix + "dead_experts": sum(u["dead_experts"] for u in util)}


def reshard_experts(shards: list[Tensor], infer_ep: int, dim: int = 0) -> list[Tensor]:
    """Stacked expert tensors of ``len(shards)`` training EP ranks (each
    [E / train_ep, ...] along ``dim``) -> ``infer_ep`` shards of
    [E / infer_ep, ...] in expert order.  Works for any widths that divide
    the expert count, narrower or wider than the training layout."""
    if infer_ep < 1 or not shards:
        raise ValueError("reshard_experts: need at least one shard and infer_ep >= 1")
    full = shards[0] if len(shards) == 1 else torch.cat(shards, dim=dim)
    E = full.shape[dim]
    if E % infer_ep:
        raise ValueError(f"reshard_experts: {E} experts do not split over {infer_ep} inference EP ranks")
    return list(torch.split(full, E // infer_ep, dim=dim))


def attach_router_stats(model, device: Optional[torch.device] = None) -> Optional[RouterStats]:
    """Give an MoE model a ``RouterStats`` (None for dense models)."""
    a = model.args
    if not getattr(a, "num_experts", 0):
        return None
    st = RouterStats(a.num_layers, a.num_experts, device or model.flat.device)
    model.router_stats = st
    return st
