"""Advantage estimators and their registry.

Estimator contract (reference ``lumenrl/algorithms/advantage_estimators.py:42-54``):
``fn(batch: DataProto, config: LumenRLConfig) -> DataProto`` writes
``batch.tensors["advantages"]`` (and ``"returns"`` where defined).

Implemented estimators (same names and math as the reference, :151-865):
``grpo``, ``dapo``, ``gae``, ``reinforce_plus_plus``, ``rloo``,
``grpo_vectorized`` (Dr.GRPO switch), ``gdpo``, ``grpo_passk``,
``reinforce_plus_plus_baseline``, ``remax``, ``opo``, ``gpg``,
``rloo_vectorized``.

Everything here is vectorised over groups (``view(-1, G)`` or scatter over a
group index) rather than per-sample python loops.  On CUDA tensors the GRPO
and DAPO normalisation runs as one fused kernel (``ops.group_advantage``).
"""

from __future__ import annotations

import logging
from typing import Callable

import torch
from torch import Tensor

from lumenrl_b200.algorithms.dapo_sampling import overlong_buffer_penalty
from lumenrl_b200.core.protocol import DataProto

logger = logging.getLogger(__name__)

ADV_ESTIMATOR_REGISTRY: dict[str, Callable] = {}


def register_adv_est(name: str) -> Callable:
    def wrap(fn: Callable) -> Callable:
        if name in ADV_ESTIMATOR_REGISTRY:
            logger.warning("Overwriting advantage estimator %r", name)
        ADV_ESTIMATOR_REGISTRY[name] = fn
        return fn
    return wrap


def get_adv_estimator(name: str) -> Callable:
    if name not in ADV_ESTIMATOR_REGISTRY:
        raise KeyError(f"no advantage estimator named {name!r}; registered: {sorted(ADV_ESTIMATOR_REGISTRY)}")
    return ADV_ESTIMATOR_REGISTRY[name]


# ---------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------

def response_mask_of(batch: DataProto) -> Tensor | None:
    for key in ("response_mask", "attention_mask"):
        if key in batch.tensors:
            return batch.tensors[key].to(torch.bool)
    return None


def _flat_rewards(batch: DataProto, what: str) -> Tensor:
    """One score per sequence: scalar rewards as they are, token-level
    rewards (e.g. after KL-in-reward shaping) summed over the response."""
    if "rewards" not in batch.tensors:
        raise KeyError(f"{what} requires tensor key 'rewards' on the batch.")
    r = batch.tensors["rewards"]
    if r.dim() > 1 and r.shape[-1] > 1:
        return r.sum(-1)
    return r.squeeze(-1) if r.dim() > 1 else r


def _group_size(batch: DataProto, config) -> int:
    return int(batch.meta.get("num_generations", config.algorithm.grpo.num_generations))


def masked_whiten(values: Tensor, mask: Tensor, shift_mean: bool = True) -> Tensor:
    """Normalise ``values`` by the mean/std of its masked entries (unbiased std,
    clamp 1e-8); fewer than two valid entries leaves ``values`` unchanged."""
    sel = values[mask.bool()]
    if sel.numel() < 2:
        return values
    centre = sel.mean() if shift_mean else 0.0
    return (values - centre) / sel.std().clamp(min=1e-8) * mask.float()


def last_token_index(mask: Tensor) -> Tensor:
    return (mask.long().sum(-1) - 1).clamp(min=0)


def scalar_to_token_rewards(rewards: Tensor, mask: Tensor) -> Tensor:
    """Place each row's scalar reward on its last valid position."""
    if rewards.dim() > 1:
        rewards = rewards.squeeze(-1)
    out = torch.zeros(mask.shape, dtype=rewards.dtype, device=mask.device)
    out[torch.arange(mask.shape[0], device=mask.device), last_token_index(mask)] = rewards.to(out.dtype)
    return out


def token_level_rewards(batch: DataProto) -> Tensor:
    r = batch.tensors["rewards"]
    if r.dim() == 1 or (r.dim() == 2 and r.shape[-1] == 1):
        return scalar_to_token_rewards(r.reshape(-1), response_mask_of(batch))
    return r


def _broadcast_to_tokens(adv: Tensor, mask: Tensor | None) -> Tensor:
    if mask is not None and mask.dim() > 1:
        return adv.unsqueeze(-1) * mask.float()
    return adv


def _group_ids(batch: DataProto, config, n: int, device) -> Tensor:
    """Per-row group index; ``uid`` meta (list of prompt ids) wins over the
    contiguous ``num_generations`` layout."""
    uids = batch.meta.get("uid")
    if uids is not None and len(uids) == n:
        mapping: dict = {}
        ids = [mapping.setdefault(u, len(mapping)) for u in uids]
        return torch.as_tensor(ids, device=device, dtype=torch.long)
    return torch.arange(n, device=device) // _group_size(batch, config)


def _segment_mean(values: Tensor, gid: Tensor, weights: Tensor | None = None) -> tuple[Tensor, Tensor]:
    """Per-row group mean (weighted if given) and per-row group count."""
    ng = int(gid.max().item()) + 1 if gid.numel() else 0
    w = torch.ones_like(values) if weights is None else weights.to(values.dtype)
    num = torch.zeros(ng, dtype=values.dtype, device=values.device).index_add_(0, gid, values * w)
    den = torch.zeros(ng, dtype=values.dtype, device=values.device).index_add_(0, gid, w)
    cnt = torch.zeros(ng, dtype=values.dtype, device=values.device).index_add_(0, gid, torch.ones_like(values))
    return (num / den.clamp(min=1e-12))[gid], cnt[gid]


def group_normalize(rewards: Tensor, group: int, unbiased: bool, eps: float = 1e-8,
                    norm_by_std: bool = True) -> Tensor:
    """(r - mean_g) / max(std_g, eps) over contiguous groups of ``group`` rows."""
    if rewards.shape[0] % group:
        raise ValueError(f"Batch size {rewards.shape[0]} not divisible by num_generations={group}.")
    if rewards.is_cuda and rewards.dtype == torch.float32 and norm_by_std:
        from lumenrl_b200.ops import group_advantage
        return group_advantage(rewards, group, unbiased=unbiased, eps=eps)
    g = rewards.view(-1, group)
    centred = g - g.mean(dim=1, keepdim=True)
    if not norm_by_std:
        return centred.reshape(-1)
    std = g.std(dim=1, unbiased=unbiased, keepdim=True).clamp_min(eps)
    return (centred / std).reshape(-1)


# ---------------------------------------------------------------------------
# estimators
# ---------------------------------------------------------------------------

@register_adv_est("grpo")
def compute_grpo_advantage(batch: DataProto, config) -> DataProto:
    """GRPO: per-group ``(r - mean) / std`` with the biased std clamped at 1e-8
    (reference ``advantage_estimators.py:151-176``)."""
    r = _flat_rewards(batch, "GRPO")
    batch.tensors["advantages"] = group_normalize(r.float(), config.algorithm.grpo.num_generations, unbiased=False)
    return batch


@register_adv_est("dapo")
def compute_dapo_advantage(batch: DataProto, config) -> DataProto:
    """DAPO: optional overlong shaping, zero-variance group mask
    (``dapo_sample_mask``), then group normalisation with the *unbiased* std
    (reference ``advantage_estimators.py:179-262``)."""
    r = _flat_rewards(batch, "DAPO").float()
    cfg = config.algorithm.dapo
    g = cfg.num_generations
    if r.shape[0] % g:
        raise ValueError(f"Batch size {r.shape[0]} not divisible by num_generations={g}.")
    lengths = batch.meta.get("response_lengths")
    ob = cfg.overlong_buffer
    if ob.enable:
        if lengths is not None:
            max_resp = int(cfg.max_resp_len) or int(config.policy.max_response_length)
            pen = overlong_buffer_penalty(lengths, max_resp, int(ob.len), float(ob.penalty_factor)).to(r.device)
            if pen.shape[0] == r.shape[0]:
                r = r + pen
    elif cfg.overlong_reward_shaping and lengths is not None:
        penalty = float(batch.meta.get("overlong_penalty", 1.0))
        lens = torch.as_tensor(lengths, device=r.device, dtype=torch.float32)
        if penalty > 0 and lens.shape[0] == r.shape[0]:
            r = r - penalty * (lens - float(config.policy.max_total_sequence_length)).clamp(min=0)
    grouped = r.view(-1, g)
    if cfg.dynamic_sampling:
        keep = grouped.std(dim=1, unbiased=False) > 1e-6
        if not bool(keep.any()):
            logger.warning("DAPO dynamic sampling removed all groups; keeping all.")
            keep = torch.ones_like(keep)
        row_mask = keep.repeat_interleave(g)
    else:
        row_mask = torch.ones(r.shape[0], dtype=torch.bool, device=r.device)
    batch.tensors["advantages"] = group_normalize(r, g, unbiased=True)
    batch.tensors["dapo_sample_mask"] = row_mask.float()
    return batch


def gae(token_rewards: Tensor, values: Tensor, mask: Tensor, gamma: float, lam: float) -> tuple[Tensor, Tensor]:
    """GAE-lambda advantages and returns; value after the last valid step is 0."""
    m = mask.to(values.dtype)
    nxt = torch.zeros_like(values)
    nxt[:, :-1] = values[:, 1:]
    last = last_token_index(mask)
    nxt[torch.arange(values.shape[0], device=values.device), last] = 0.0
    delta = token_rewards + gamma * nxt * m - values
    adv = torch.zeros_like(delta)
    run = torch.zeros(values.shape[0], device=values.device, dtype=values.dtype)
    for t in range(delta.shape[1] - 1, -1, -1):
        run = delta[:, t] + gamma * lam * m[:, t] * run
        adv[:, t] = run
    ret = adv + values
    return adv * m, ret * m


@register_adv_est("gae")
def compute_gae_advantage(batch: DataProto, config) -> DataProto:
    if "values" not in batch.tensors:
        raise KeyError("GAE requires critic 'values' tensor [B, T].")
    if "rewards" not in batch.tensors:
        raise KeyError("GAE requires 'rewards' (scalar or token-level).")
    mask = response_mask_of(batch)
    if mask is None:
        raise KeyError("GAE requires 'response_mask' or 'attention_mask' for masking.")
    values = batch.tensors["values"]
    tr = token_level_rewards(batch).to(values.dtype)
    if tr.shape != values.shape:
        raise ValueError(f"Token rewards shape {tuple(tr.shape)} != values {tuple(values.shape)}.")
    cfg = config.algorithm.ppo
    adv, ret = gae(tr, values, mask.float(), float(cfg.discount), float(cfg.gae_lambda))
    batch.tensors["advantages"], batch.tensors["returns"] = adv, ret
    return batch


@register_adv_est("reinforce_plus_plus")
def compute_reinforce_plus_plus_advantage(batch: DataProto, config) -> DataProto:
    r = _flat_rewards(batch, "REINFORCE++")
    mask = response_mask_of(batch)
    if mask is None:
        raise KeyError("REINFORCE++ requires 'response_mask' or 'attention_mask'.")
    mf = mask.float()
    tr = scalar_to_token_rewards(r, mask)
    gamma = float(config.algorithm.ppo.discount)
    ret = torch.zeros_like(tr)
    run = torch.zeros(tr.shape[0], dtype=tr.dtype, device=tr.device)
    for t in range(tr.shape[1] - 1, -1, -1):
        run = tr[:, t] + gamma * run * mf[:, t]
        ret[:, t] = run
    batch.tensors["advantages"] = masked_whiten(ret, mf)
    return batch


@register_adv_est("rloo")
def compute_rloo_advantage(batch: DataProto, config) -> DataProto:
    r = _flat_rewards(batch, "RLOO")
    g = _group_size(batch, config)
    if r.shape[0] % g:
        raise ValueError(f"Batch size {r.shape[0]} not divisible by num_generations={g}.")
    mask = response_mask_of(batch)
    if mask is None:
        raise KeyError("RLOO requires 'response_mask' or 'attention_mask'.")
    grouped = r.view(-1, g)
    loo = grouped - (grouped.sum(1, keepdim=True) - grouped) / (g - 1.0)
    tok = loo.reshape(-1, 1) * mask.float()
    batch.tensors["advantages"] = masked_whiten(tok, mask.float())
    return batch


@register_adv_est("grpo_vectorized")
def compute_grpo_vectorized_advantage(batch: DataProto, config) -> DataProto:
    """GRPO with the Dr.GRPO switch ``meta['norm_adv_by_std_in_grpo']``."""
    r = _flat_rewards(batch, "GRPO").float()
    adv = group_normalize(r, config.algorithm.grpo.num_generations, unbiased=False,
                          norm_by_std=bool(batch.meta.get("norm_adv_by_std_in_grpo", True)))
    batch.tensors["advantages"] = _broadcast_to_tokens(adv, response_mask_of(batch))
    return batch


@register_adv_est("gdpo")
def compute_gdpo_advantage(batch: DataProto, config) -> DataProto:
    """Group reward-decoupled normalisation: each reward component is group
    normalised on its own, summed, then whitened over response tokens."""
    mask = response_mask_of(batch)
    g = config.algorithm.grpo.num_generations
    comps = batch.tensors.get("reward_components")
    if comps is None:
        tr = token_level_rewards(batch)
        comps = (tr.sum(-1) if tr.dim() > 1 else tr).unsqueeze(-1)
    total = None
    for j in range(comps.shape[-1]):
        n = group_normalize(comps[:, j].float(), g, unbiased=False)
        n = _broadcast_to_tokens(n, mask)
        total = n if total is None else total + n
    if mask is not None and mask.dim() > 1:
        total = masked_whiten(total, mask.float()) * mask.float()
    batch.tensors["advantages"] = total
    return batch


@register_adv_est("grpo_passk")
def compute_grpo_passk_advantage(batch: DataProto, config) -> DataProto:
    """Pass@k: only each group's best sample gets ``(top1 - top2) / std``."""
    r = _flat_rewards(batch, "GRPO pass@k").float()
    gid = _group_ids(batch, config, r.shape[0], r.device)
    adv = torch.zeros_like(r)
    for gi in torch.unique(gid).tolist():
        rows = (gid == gi).nonzero(as_tuple=True)[0]
        if rows.numel() < 2:
            continue
        vals = r[rows]
        top, pos = torch.topk(vals, 2)
        adv[rows[pos[0]]] = (top[0] - top[1]) / vals.std().clamp_min(1e-8)
    batch.tensors["advantages"] = _broadcast_to_tokens(adv, response_mask_of(batch))
    return batch


def _group_mean_baseline(r: Tensor, gid: Tensor) -> Tensor:
    mean, cnt = _segment_mean(r, gid)
    return torch.where(cnt > 1, mean, torch.zeros_like(mean))


@register_adv_est("reinforce_plus_plus_baseline")
def compute_reinforce_pp_baseline_advantage(batch: DataProto, config) -> DataProto:
    r = _flat_rewards(batch, "RF++ baseline").float()
    gid = _group_ids(batch, config, r.shape[0], r.device)
    s = r - _group_mean_baseline(r, gid)
    mask = response_mask_of(batch)
    if mask is not None and mask.dim() > 1:
        mf = mask.float()
        s = masked_whiten(s.unsqueeze(-1) * mf, mf) * mf
    batch.tensors["advantages"] = s
    return batch


@register_adv_est("remax")
def compute_remax_advantage(batch: DataProto, config) -> DataProto:
    tr = token_level_rewards(batch)
    mask = response_mask_of(batch)
    mf = mask.float() if mask is not None else torch.ones_like(tr)
    base = batch.tensors.get("reward_baselines")
    if base is None:
        base = torch.zeros(tr.shape[0], device=tr.device)
    base = base.reshape(-1)
    ret = (tr * mf).flip(-1).cumsum(-1).flip(-1)
    batch.tensors["advantages"] = ret - base.unsqueeze(-1) * mf
    batch.tensors["returns"] = ret
    return batch


@register_adv_est("opo")
def compute_opo_advantage(batch: DataProto, config) -> DataProto:
    """Length-weighted group baseline (OPO)."""
    r = _flat_rewards(batch, "OPO").float()
    gid = _group_ids(batch, config, r.shape[0], r.device)
    mask = response_mask_of(batch)
    lens = mask.float().sum(-1) if mask is not None and mask.dim() > 1 else torch.ones_like(r)
    mean, cnt = _segment_mean(r, gid, weights=lens)
    s = r - torch.where(cnt > 1, mean, torch.zeros_like(mean))
    batch.tensors["advantages"] = _broadcast_to_tokens(s, mask)
    return batch


@register_adv_est("gpg")
def compute_gpg_advantage(batch: DataProto, config) -> DataProto:
    r = _flat_rewards(batch, "GPG").float()
    gid = _group_ids(batch, config, r.shape[0], r.device)
    alpha = float(r.shape[0]) / max(int(torch.count_nonzero(r).item()), 1)
    s = alpha * (r - _group_mean_baseline(r, gid))
    batch.tensors["advantages"] = _broadcast_to_tokens(s, response_mask_of(batch))
    return batch


@register_adv_est("rloo_vectorized")
def compute_rloo_vectorized_advantage(batch: DataProto, config) -> DataProto:
    r = _flat_rewards(batch, "RLOO").float()
    gid = _group_ids(batch, config, r.shape[0], r.device)
    ng = int(gid.max().item()) + 1
    cnt = torch.bincount(gid, minlength=ng)[gid].float()
    tot = torch.zeros(ng, device=r.device, dtype=r.dtype).index_add_(0, gid, r)[gid]
    adv = (cnt * r - tot) / (cnt - 1).clamp_min(1) * (cnt > 1)
    batch.tensors["advantages"] = _broadcast_to_tokens(adv, response_mask_of(batch))
    return batch
