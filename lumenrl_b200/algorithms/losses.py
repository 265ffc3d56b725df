"""Policy-optimisation loss library (reference ``lumenrl/algorithms/loss_functions.py:30-457``).

Same function names, arguments and maths as the reference (the verl loss
conventions are the public contract that recipes are tuned against):

* ``agg_loss``: token-mean / seq-mean-token-sum(-norm) / seq-mean-token-mean,
  with the global-token (``batch_num_tokens``) and ``dp_size`` compensation
  used under data parallelism.
* ``policy_gradient_loss``: symmetric PPO clip, masked mean.
* ``asymmetric_clip_loss``: DAPO clip-higher + dual clip + TIS weights +
  global-token normalisation.  On CUDA the per-token part runs as the fused
  ``ops.ppo_clip_loss`` kernel (forward and backward in one pass each).
* ``gmpo_loss``, ``value_loss``, ``kl_penalty``, ``opd_kl_divergence``,
  ``hidden_state_loss``, ``entropy_bonus``, ``sft_loss``.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn.functional as F
from torch import Tensor

__all__ = [
    "agg_loss", "sft_loss", "policy_gradient_loss", "asymmetric_clip_loss", "gmpo_loss",
    "value_loss", "kl_penalty", "opd_kl_divergence", "hidden_state_loss", "entropy_bonus",
    "masked_sum", "masked_mean",
]


def masked_sum(values: Tensor, mask: Tensor, dim=None) -> Tensor:
    v = torch.where(mask.bool(), values, torch.zeros_like(values))
    return v.sum() if dim is None else v.sum(dim=dim)


def masked_mean(values: Tensor, mask: Tensor, dim=None) -> Tensor:
    m = mask.to(values.dtype)
    return masked_sum(values, mask, dim) / (m.sum() if dim is None else m.sum(dim=dim)).clamp(min=1e-8)


def _masked_avg(x: Tensor, mask: Optional[Tensor]) -> Tensor:
    if mask is None:
        return x.mean()
    w = mask.to(x.dtype)
    return (x * w).sum() / w.sum().clamp(min=1.0)


def agg_loss(loss_mat: Tensor, loss_mask: Tensor, loss_agg_mode: str, dp_size: int = 1,
             batch_num_tokens: Optional[int] = None, global_batch_size: Optional[int] = None) -> Tensor:
    if loss_agg_mode == "token-mean":
        if batch_num_tokens is None:
            if dp_size > 1:
                raise ValueError("batch_num_tokens is required when dp_size > 1")
            batch_num_tokens = int(loss_mask.sum().item())
        return masked_sum(loss_mat, loss_mask) / max(batch_num_tokens, 1) * dp_size
    if loss_agg_mode in ("seq-mean-token-sum", "seq-mean-token-sum-norm", "seq-mean-token-mean"):
        m = loss_mask.to(loss_mat.dtype)
        tok = m.sum(-1)
        per_seq = (loss_mat * m).sum(-1)
        if loss_agg_mode == "seq-mean-token-mean":
            per_seq = per_seq / (tok + 1e-8)
        seq_mask = (tok > 0).float()
        if global_batch_size is None:
            if dp_size > 1:
                raise ValueError("global_batch_size is required when dp_size > 1")
            global_batch_size = int(seq_mask.sum().item())
        out = masked_sum(per_seq, seq_mask) / max(global_batch_size, 1) * dp_size
        if loss_agg_mode == "seq-mean-token-sum-norm":
            out = out / loss_mask.shape[-1]
        return out
    raise ValueError(f"Invalid loss_agg_mode: {loss_agg_mode!r}")


def sft_loss(log_probs: Tensor, loss_mask: Tensor, loss_agg_mode: str = "token-mean",
             dp_size: int = 1, dp_group=None) -> tuple[Tensor, dict[str, float]]:
    import torch.distributed as dist
    bnt = gbs = None
    if loss_agg_mode == "token-mean":
        n = loss_mask.sum().float()
        if dp_group is not None and dist.is_initialized():
            dist.all_reduce(n, group=dp_group)
        bnt = max(int(n.item()), 1)
    else:
        n = (loss_mask.sum(-1) > 0).float().sum()
        if dp_group is not None and dist.is_initialized():
            dist.all_reduce(n, group=dp_group)
        gbs = max(int(n.item()), 1)
    loss = agg_loss(-log_probs, loss_mask, loss_agg_mode, dp_size=dp_size,
                    batch_num_tokens=bnt, global_batch_size=gbs)
    return loss, {"sft_loss": float(loss.detach()), "num_tokens": float(loss_mask.sum().detach())}


def policy_gradient_loss(logprobs: Tensor, old_logprobs: Tensor, advantages: Tensor, clip_ratio: float,
                         *, mask: Optional[Tensor] = None) -> Tensor:
    ratio = torch.exp(logprobs - old_logprobs)
    pg = -torch.minimum(ratio * advantages, ratio.clamp(1.0 - clip_ratio, 1.0 + clip_ratio) * advantages)
    return _masked_avg(pg, mask)


def asymmetric_clip_token_losses(logprobs: Tensor, old_logprobs: Tensor, advantages: Tensor,
                                 clip_low: float, clip_high: float, clip_ratio_c: float = 0.0,
                                 rollout_is_weights: Optional[Tensor] = None) -> Tensor:
    """Per-token DAPO surrogate (before masking / aggregation)."""
    ratio = torch.exp((logprobs - old_logprobs).clamp(-20.0, 20.0))
    pg = torch.maximum(-advantages * ratio, -advantages * ratio.clamp(1.0 - clip_low, 1.0 + clip_high))
    if clip_ratio_c > 0.0:
        pg = torch.where(advantages < 0, torch.minimum(-advantages * clip_ratio_c, pg), pg)
    if rollout_is_weights is not None:
        pg = pg * rollout_is_weights.to(pg.dtype)
    return pg


def asymmetric_clip_loss(logprobs: Tensor, old_logprobs: Tensor, advantages: Tensor, clip_low: float,
                         clip_high: float, *, mask: Optional[Tensor] = None, clip_ratio_c: float = 0.0,
                         batch_num_tokens: Optional[int] = None, dp_size: int = 1,
                         rollout_is_weights: Optional[Tensor] = None) -> Tensor:
    if logprobs.is_cuda and mask is not None and logprobs.dtype == torch.float32:
        from lumenrl_b200.ops import ppo_clip_loss
        denom = float(max(batch_num_tokens, 1)) / dp_size if batch_num_tokens is not None else None
        return ppo_clip_loss(logprobs, old_logprobs, advantages, mask, clip_low, clip_high, clip_ratio_c,
                             rollout_is_weights, denom)
    pg = asymmetric_clip_token_losses(logprobs, old_logprobs, advantages, clip_low, clip_high,
                                      clip_ratio_c, rollout_is_weights)
    if mask is None:
        return pg.mean()
    pg = torch.where(mask.bool(), pg, torch.zeros_like(pg))
    if batch_num_tokens is not None:
        return pg.sum() / max(batch_num_tokens, 1) * dp_size
    return pg.sum() / mask.to(pg.dtype).sum().clamp(min=1.0)


def gmpo_loss(logprobs: Tensor, old_logprobs: Tensor, advantages: Tensor, clip_low: float, clip_high: float,
              *, mask: Optional[Tensor] = None) -> Tensor:
    """Geometric-mean PO: clip the per-token log-ratio toward zero on the side
    the advantage sign makes harmful, geometric-mean it per sequence."""
    lr = logprobs - old_logprobs
    s = torch.sign(advantages)
    lr_clipped = s * torch.minimum(s * lr, s * lr.clamp(-clip_low, clip_high))
    if mask is not None:
        w = mask.to(lr_clipped.dtype)
        n = w.sum(-1)
        ratio = torch.exp((lr_clipped * w).sum(-1) / (n + 1e-8))
        seq_adv = (advantages * w).sum(-1) / (n + 1e-8)
    else:
        ratio = torch.exp(lr_clipped.mean(-1))
        seq_adv = advantages.mean(-1)
    return (-seq_adv * ratio).mean()


def value_loss(values: Tensor, old_values: Tensor, returns: Tensor, clip_ratio: float,
               *, mask: Optional[Tensor] = None) -> Tensor:
    clipped = old_values + (values - old_values).clamp(-clip_ratio, clip_ratio)
    vf = torch.maximum((values - returns) ** 2, (clipped - returns) ** 2)
    return _masked_avg(vf, mask)


def kl_penalty(logprobs: Tensor, ref_logprobs: Tensor, *, mask: Optional[Tensor] = None) -> Tensor:
    return _masked_avg(ref_logprobs - logprobs, mask)


def opd_kl_divergence(student_logits: Tensor, teacher_logits: Tensor, *, mask: Optional[Tensor] = None,
                      kl_direction: str = "reverse", temperature: float = 1.0,
                      position_weights: Optional[Tensor] = None) -> Tensor:
    if temperature != 1.0:
        student_logits = student_logits / temperature
        teacher_logits = teacher_logits / temperature
    ls = F.log_softmax(student_logits.float(), dim=-1)
    lt = F.log_softmax(teacher_logits.float(), dim=-1)
    if kl_direction == "reverse":
        kl = (ls.exp() * (ls - lt)).sum(-1)
    elif kl_direction == "forward":
        kl = (lt.exp() * (lt - ls)).sum(-1)
    else:
        raise ValueError(f"Unknown kl_direction: {kl_direction!r}. Use 'reverse' or 'forward'.")
    if position_weights is not None:
        pw = position_weights[: kl.shape[1]].to(kl.dtype).to(kl.device)
        kl = kl * pw.unsqueeze(0)
    return _masked_avg(kl, mask)


def hidden_state_loss(student_hidden: Tensor, teacher_hidden: Tensor, *, mask: Optional[Tensor] = None,
                      loss_type: str = "mse", projection: Optional[torch.nn.Module] = None) -> Tensor:
    if projection is not None:
        student_hidden = projection(student_hidden)
    if loss_type == "mse":
        per = ((student_hidden.float() - teacher_hidden.float()) ** 2).mean(-1)
    elif loss_type == "cosine":
        per = 1.0 - F.cosine_similarity(student_hidden.float(), teacher_hidden.float(), dim=-1)
    else:
        raise ValueError(f"Unknown loss_type: {loss_type!r}. Use 'mse' or 'cosine'.")
    return _masked_avg(per, mask)


def entropy_bonus(logprobs: Tensor, *, mask: Optional[Tensor] = None) -> Tensor:
    return _masked_avg(-(torch.exp(logprobs) * logprobs), mask)
