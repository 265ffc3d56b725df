"""GRPO (reference ``lumenrl/algorithms/grpo.py:34-71``): group-normalised
scalar advantages, symmetric PPO clip, optional ``kl_coeff * KL(ref)``."""

from __future__ import annotations

from typing import Any

from torch import Tensor

from lumenrl_b200.algorithms.base import BaseAlgorithm, expand_to_tokens, response_mask
from lumenrl_b200.algorithms.losses import kl_penalty, policy_gradient_loss
from lumenrl_b200.core.protocol import DataProto
from lumenrl_b200.core.registry import ALGORITHM_REGISTRY


class GRPOAlgorithm(BaseAlgorithm):
    def compute_loss(self, batch: DataProto) -> tuple[Tensor, dict[str, Any]]:
        t = batch.tensors
        if "log_probs" not in t or "old_log_probs" not in t:
            raise KeyError("GRPO loss requires 'log_probs' and 'old_log_probs'.")
        if "advantages" not in t:
            raise KeyError("GRPO loss requires precomputed 'advantages'.")
        mask = response_mask(batch)
        logp = t["log_probs"]
        adv = expand_to_tokens(t["advantages"], logp, mask)
        cfg = self._config.algorithm.grpo
        pg = policy_gradient_loss(logp, t["old_log_probs"], adv, cfg.clip_ratio, mask=mask)
        loss, metrics = pg, {"loss_pg": float(pg.detach())}
        if cfg.kl_coeff > 0.0 and "ref_log_probs" in t:
            kl = kl_penalty(logp, t["ref_log_probs"], mask=mask)
            loss = loss + cfg.kl_coeff * kl
            metrics["kl"] = float(kl.detach())
        metrics["loss_total"] = float(loss.detach())
        return loss, metrics


ALGORITHM_REGISTRY.register("grpo", GRPOAlgorithm)
