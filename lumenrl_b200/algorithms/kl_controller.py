"""KL controllers and KL-in-reward (reference ``lumenrl/algorithms/kl_controller.py:28-170``).

* ``FixedKLController`` / ``AdaptiveKLController`` (proportional controller
  with the error clipped to +-0.2, Ziegler et al. 2019).
* ``kl_penalty_forward``: estimators ``kl``/``k1``, ``abs``, ``mse``/``k2``,
  ``low_var_kl``/``k3`` (k3 clamped to [-10, 10]).
* ``kl_penalty_token``: a trailing ``+`` keeps the forward value but takes the
  k2 gradient (straight-through).
* ``apply_kl_penalty``: token rewards ``r - beta * KL`` and controller update.
"""

from __future__ import annotations

from typing import Any

import torch
from torch import Tensor

from lumenrl_b200.core.protocol import DataProto


class AdaptiveKLController:
    def __init__(self, init_kl_coef: float, target_kl: float, horizon: int) -> None:
        self.value = float(init_kl_coef)
        self.target = float(target_kl)
        self.horizon = int(horizon)

    def update(self, current_kl: float, n_steps: int) -> None:
        err = min(max(current_kl / self.target - 1.0, -0.2), 0.2)
        self.value *= 1.0 + err * n_steps / self.horizon


class FixedKLController:
    def __init__(self, kl_coef: float) -> None:
        self.value = float(kl_coef)

    def update(self, current_kl: float, n_steps: int) -> None:
        return None


def get_kl_controller(kl_ctrl_type: str, kl_coef: float, target_kl: float = 0.01, horizon: int = 10000):
    if kl_ctrl_type == "fixed":
        return FixedKLController(kl_coef)
    if kl_ctrl_type == "adaptive":
        if horizon <= 0:
            raise ValueError(f"horizon must be > 0, got {horizon}")
        return AdaptiveKLController(kl_coef, target_kl, horizon)
    raise ValueError(f"Unknown kl_ctrl_type: {kl_ctrl_type!r}. Use 'fixed' or 'adaptive'.")


def kl_penalty_forward(logprob: Tensor, ref_logprob: Tensor, kl_penalty_type: str) -> Tensor:
    d = logprob - ref_logprob
    if kl_penalty_type in ("kl", "k1"):
        return d
    if kl_penalty_type == "abs":
        return d.abs()
    if kl_penalty_type in ("mse", "k2"):
        return 0.5 * d * d
    if kl_penalty_type in ("low_var_kl", "k3"):
        x = (-d).clamp(-20.0, 20.0)
        return (torch.exp(x) - x - 1.0).clamp(-10.0, 10.0)
    raise NotImplementedError(f"Unknown kl_penalty type: {kl_penalty_type!r}")


def kl_penalty_token(logprob: Tensor, ref_logprob: Tensor, kl_penalty_type: str) -> Tensor:
    base = kl_penalty_type.rstrip("+")
    fwd = kl_penalty_forward(logprob, ref_logprob, base)
    if not kl_penalty_type.endswith("+") or kl_penalty_type in ("mse", "k2"):
        return fwd
    k2 = 0.5 * (logprob - ref_logprob) ** 2
    return k2 - k2.detach() + fwd.detach()


def masked_mean(values: Tensor, mask: Tensor, axis: int = -1) -> Tensor:
    return (values * mask).sum(dim=axis) / mask.sum(dim=axis).clamp(min=1.0)


def apply_kl_penalty(batch: DataProto, kl_ctrl, kl_penalty_type: str = "kl") -> tuple[DataProto, dict[str, Any]]:
    from lumenrl_b200.algorithms.advantage import response_mask_of, scalar_to_token_rewards
    mask = batch.tensors.get("response_mask", batch.tensors.get("attention_mask"))
    if mask is None:
        raise KeyError("apply_kl_penalty requires 'response_mask' or 'attention_mask'.")
    mf = mask.float()
    kld = kl_penalty_token(batch.tensors["old_log_probs"], batch.tensors["ref_log_probs"], kl_penalty_type) * mf
    r = batch.tensors["rewards"]
    if r.dim() == 1 or (r.dim() == 2 and r.shape[-1] == 1):
        tok = scalar_to_token_rewards(r.reshape(-1), response_mask_of(batch))
    else:
        tok = r.float()
    beta = kl_ctrl.value
    current = masked_mean(kld, mf, axis=-1).mean().item()
    kl_ctrl.update(current_kl=current, n_steps=batch.tensors["old_log_probs"].shape[0])
    batch.tensors["rewards"] = tok - beta * kld
    batch.tensors["token_level_scores"] = tok
    batch.meta["kl_penalty_applied"] = True
    return batch, {"actor/reward_kl_penalty": current, "actor/reward_kl_penalty_coeff": beta}
