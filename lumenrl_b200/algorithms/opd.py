"""On-policy distillation (reference ``lumenrl/algorithms/opd.py:33-85``):
full-vocabulary KL(student||teacher) (or forward), temperature, optional
``decay**position`` weights; no reward-based advantages."""

from __future__ import annotations

from typing import Any

import torch
from torch import Tensor

from lumenrl_b200.algorithms.base import BaseAlgorithm, response_mask
from lumenrl_b200.algorithms.losses import opd_kl_divergence
from lumenrl_b200.core.protocol import DataProto
from lumenrl_b200.core.registry import ALGORITHM_REGISTRY


class OPDAlgorithm(BaseAlgorithm):
    def compute_advantages(self, batch: DataProto) -> DataProto:
        return batch

    def compute_loss(self, batch: DataProto) -> tuple[Tensor, dict[str, Any]]:
        for k in ("student_logits", "teacher_logits"):
            if k not in batch.tensors:
                raise KeyError(f"OPD requires '{k}' on the batch.")
        cfg = self._config.algorithm.opd
        pw = None
        if cfg.position_weighting:
            n = batch["student_logits"].shape[1]
            pw = cfg.position_decay ** torch.arange(n, dtype=torch.float32)
        kl = opd_kl_divergence(batch["student_logits"], batch["teacher_logits"].detach(), mask=response_mask(batch),
                               kl_direction=cfg.kl_direction, temperature=cfg.temperature, position_weights=pw)
        loss = cfg.opd_coeff * kl
        return loss, {"opd_kl": float(kl.detach()), "loss_total": float(loss.detach())}

    def get_config(self) -> dict[str, Any]:
        import dataclasses
        return {"name": self._config.algorithm.name, "opd": dataclasses.asdict(self._config.algorithm.opd)}


ALGORITHM_REGISTRY.register("opd", OPDAlgorithm)
