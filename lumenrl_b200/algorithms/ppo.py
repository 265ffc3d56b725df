"""PPO (reference ``lumenrl/algorithms/ppo.py:17-69``): clipped surrogate +
``0.5 *`` clipped value loss + optional KL; GAE advantages by default."""

from __future__ import annotations

from typing import Any

import torch
from torch import Tensor

from lumenrl_b200.algorithms.base import BaseAlgorithm
from lumenrl_b200.algorithms.losses import kl_penalty, policy_gradient_loss, value_loss
from lumenrl_b200.core.protocol import DataProto
from lumenrl_b200.core.registry import ALGORITHM_REGISTRY


class PPOAlgorithm(BaseAlgorithm):
    def compute_loss(self, batch: DataProto) -> tuple[Tensor, dict[str, Any]]:
        t = batch.tensors
        for k in ("log_probs", "old_log_probs", "advantages", "values", "returns"):
            if k not in t:
                raise KeyError(f"PPO loss missing tensor '{k}'.")
        adv = t["advantages"]
        m = t.get("attention_mask")
        mask = torch.ones_like(adv) if m is None else m.to(adv.dtype)
        cfg = self._config.algorithm.ppo
        pg = policy_gradient_loss(t["log_probs"], t["old_log_probs"], adv, cfg.clip_ratio, mask=mask)
        values, rets = t["values"], t["returns"]
        vf = value_loss(values, t.get("old_values", values.detach()), rets, cfg.clip_ratio, mask=mask)
        loss = pg + 0.5 * vf
        metrics: dict[str, Any] = {"loss_pg": float(pg.detach()), "loss_vf": float(vf.detach())}
        if cfg.kl_coeff > 0.0 and "ref_log_probs" in t:
            kl = kl_penalty(t["log_probs"], t["ref_log_probs"], mask=mask.bool())
            loss = loss + cfg.kl_coeff * kl
            metrics["kl"] = float(kl.detach())
        with torch.no_grad():
            b = mask.bool()
            if bool(b.any()):
                ev = 1.0 - ((values[b] - rets[b]) ** 2).mean() / rets[b].float().var().clamp_min(1e-8)
                metrics["explained_variance"] = float(ev)
            else:
                metrics["explained_variance"] = 0.0
        metrics["loss_total"] = float(loss.detach())
        return loss, metrics


ALGORITHM_REGISTRY.register("ppo", PPOAlgorithm)
