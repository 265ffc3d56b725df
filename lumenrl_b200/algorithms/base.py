"""Algorithm interface (reference ``lumenrl/algorithms/base_algorithm.py:17-63``).

``compute_advantages`` resolves an estimator from ``algorithm.adv_estimator``
or the algorithm name (grpo->grpo, dapo->dapo, ppo->gae, opd->grpo);
``compute_loss`` returns ``(scalar_loss, metrics)``.
"""

from __future__ import annotations

import dataclasses
from abc import ABC, abstractmethod
from typing import Any

import torch
from torch import Tensor

from lumenrl_b200.core.protocol import DataProto

_DEFAULT_ESTIMATOR = {"grpo": "grpo", "dapo": "dapo", "ppo": "gae", "opd": "grpo"}


def response_mask(batch: DataProto) -> Tensor | None:
    for key in ("response_mask", "attention_mask"):
        if key in batch.tensors:
            return batch.tensors[key].to(torch.bool)
    return None


def expand_to_tokens(adv: Tensor, like: Tensor, mask: Tensor | None) -> Tensor:
    if adv.dim() == 1:
        adv = adv.unsqueeze(-1)
    adv = adv.expand_as(like)
    return adv * mask.to(adv.dtype) if mask is not None else adv


class BaseAlgorithm(ABC):
    def __init__(self, config) -> None:
        self._config = config

    @property
    def config(self):
        return self._config

    def resolve_estimator(self) -> str:
        explicit = self._config.algorithm.adv_estimator
        if explicit:
            return explicit
        return _DEFAULT_ESTIMATOR.get(self._config.algorithm.name.lower(), "grpo")

    _resolve_estimator = resolve_estimator

    def compute_advantages(self, batch: DataProto) -> DataProto:
        from lumenrl_b200.algorithms.advantage import get_adv_estimator
        return get_adv_estimator(self.resolve_estimator())(batch, self._config)

    @abstractmethod
    def compute_loss(self, batch: DataProto) -> tuple[Tensor, dict[str, Any]]:
        ...

    def get_config(self) -> dict[str, Any]:
        a = self._config.algorithm
        return {"name": a.name, **{k: dataclasses.asdict(getattr(a, k))
                                   for k in ("grpo", "dapo", "ppo", "opd", "spec_distill")}}
