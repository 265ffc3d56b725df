"""DAPO (reference ``lumenrl/algorithms/dapo.py:23-126``): clip-higher
``[1-eps_low, 1+eps_high]``, dual clip ``c``, TIS weights, global-token
normalisation; ``loss_mode`` token_level (default), sequence level, or gmpo."""

from __future__ import annotations

from typing import Any

import torch
from torch import Tensor

from lumenrl_b200.algorithms.advantage import compute_dapo_advantage
from lumenrl_b200.algorithms.base import BaseAlgorithm, expand_to_tokens, response_mask
from lumenrl_b200.algorithms.losses import asymmetric_clip_loss, gmpo_loss, kl_penalty
from lumenrl_b200.core.protocol import DataProto
from lumenrl_b200.core.registry import ALGORITHM_REGISTRY


class DAPOAlgorithm(BaseAlgorithm):
    def compute_advantages(self, batch: DataProto) -> DataProto:
        return compute_dapo_advantage(batch, self._config)

    def compute_loss(self, batch: DataProto) -> tuple[Tensor, dict[str, Any]]:
        t = batch.tensors
        if "log_probs" not in t or "old_log_probs" not in t:
            raise KeyError("DAPO loss requires 'log_probs' and 'old_log_probs'.")
        if "advantages" not in t:
            raise KeyError("DAPO loss requires 'advantages'.")
        logp, old = t["log_probs"], t["old_log_probs"]
        mask = response_mask(batch)
        adv = expand_to_tokens(t["advantages"], logp, mask)
        sm = t.get("dapo_sample_mask")
        if sm is not None:
            sm = (sm.unsqueeze(-1) if sm.dim() == 1 else sm).expand_as(logp).to(logp.dtype)
            if mask is not None:
                sm = sm * mask.to(logp.dtype)
        else:
            sm = mask.to(logp.dtype) if mask is not None else torch.ones_like(logp)
        cfg = self._config.algorithm.dapo
        ris = t.get("rollout_is_weights")
        if ris is not None:
            ris = ris.unsqueeze(-1) if ris.dim() == 1 else ris
            try:
                ris = ris.expand_as(logp)
            except RuntimeError:
                ris = None
        lo, hi, c = float(cfg.clip_ratio_low), float(cfg.clip_ratio_high), float(cfg.clip_ratio_c)
        if cfg.loss_mode == "gmpo":
            pg = gmpo_loss(logp, old, adv, lo, hi, mask=sm)
        elif cfg.token_level_pg:
            pg = asymmetric_clip_loss(logp, old, adv, lo, hi, mask=sm, clip_ratio_c=c,
                                      batch_num_tokens=batch.meta.get("batch_num_tokens"),
                                      dp_size=batch.meta.get("dp_size", 1), rollout_is_weights=ris)
        else:
            n = sm.sum(-1, keepdim=True).clamp(min=1.0)
            pg = asymmetric_clip_loss((logp * sm).sum(-1, keepdim=True) / n, (old * sm).sum(-1, keepdim=True) / n,
                                      adv.sum(-1, keepdim=True) / n, lo, hi, mask=None, clip_ratio_c=c)
        loss, metrics = pg, {"loss_pg": float(pg.detach())}
        if cfg.kl_coeff > 0.0 and "ref_log_probs" in t:
            kl = kl_penalty(logp, t["ref_log_probs"], mask=mask)
            loss = loss + cfg.kl_coeff * kl
            metrics["kl"] = float(kl.detach())
        metrics["loss_total"] = float(loss.detach())
        return loss, metrics


ALGORITHM_REGISTRY.register("dapo", DAPOAlgorithm)
