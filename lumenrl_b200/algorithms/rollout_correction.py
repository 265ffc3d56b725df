"""Rollout correction: TIS / MIS / IcePop importance weights, rejection
sampling, off-policy diagnostics and bypass mode.

Semantics follow ``lumenrl/algorithms/rollout_correction.py:43-872`` (itself
the verl ``rollout_corr_helper``):

* ``log_ratio = old_log_prob - rollout_log_prob`` (training vs rollout policy).
* IS weights at ``token`` or ``sequence`` level (sum or mean of log-ratios),
  clamped to ``upper`` (TIS) or zeroed outside ``[lower, upper]`` (IcePop,
  threshold written ``"lower_upper"``), optional batch normalisation.
* Rejection sampling over the eleven criteria
  ``token_k{1,2,3}``, ``seq_sum_k{1,2,3}``, ``seq_mean_k{1,2,3}``,
  ``seq_max_k{2,3}``; k1 takes a ``lower_upper`` ratio band (its statistic is
  ``-log_ratio``), k2/k3 an upper bound.
* Off-policy metrics: kl, k3_kl, training/rollout ppl, chi^2 token and seq.
* Rollout log-probs that are exactly 0.0 on a response position are treated as
  "not reported" and replaced by the training log-prob (de-aliasing rule).
* Legacy advantage-level TIS/MIS and the preset factories.

All statistics use masked reductions; every log-ratio is clamped to +-20
before exponentiation.
"""

from __future__ import annotations

import logging
import math
from typing import Any, Optional

import torch
from torch import Tensor

from lumenrl_b200.core.config import LumenRLConfig, QuantizationConfig, RolloutCorrectionConfig
from lumenrl_b200.core.protocol import DataProto

logger = logging.getLogger(__name__)

SAFETY_BOUND = 20.0
SUPPORTED_ROLLOUT_RS_OPTIONS = {
    "token_k1", "token_k2", "token_k3",
    "seq_sum_k1", "seq_sum_k2", "seq_sum_k3",
    "seq_mean_k1", "seq_mean_k2", "seq_mean_k3",
    "seq_max_k2", "seq_max_k3",
}
TOKEN_LEVEL_ROLLOUT_RS_OPTIONS = {"token_k1", "token_k2", "token_k3"}


class _Masked:
    """Reductions restricted to positions where the mask is non-zero
    (masked-out entries may hold inf / nan and never reach the result)."""

    @staticmethod
    def total(values: Tensor, mask: Tensor, dim=None) -> Tensor:
        kept = values.masked_fill(~mask.bool(), 0.0) * mask
        return kept.sum() if dim is None else kept.sum(dim=dim)

    @staticmethod
    def mean(values: Tensor, mask: Tensor, dim=None) -> Tensor:
        count = mask.sum() if dim is None else mask.sum(dim=dim)
        return _Masked.total(values, mask, dim) / count.clamp(min=1e-8)


_msum, _mmean = _Masked.total, _Masked.mean


# ---------------------------------------------------------------------------
# threshold grammar, shared by the IS weights and every rejection criterion:
#
#     threshold := NUMBER                 an upper bound
#                | NUMBER "_" NUMBER      a "lower_upper" band
#
# IS weights accept both (a band selects IcePop); k1 rejection criteria
# accept both (a bare NUMBER x means the band 1/x .. x); k2 / k3 criteria
# accept only an upper bound.  Every bound must be positive, lower <= upper.
# ---------------------------------------------------------------------------

def _read_bound(text: str, where: str) -> tuple[Optional[float], float]:
    """One threshold token -> (lower or None, upper)."""
    pieces = text.split("_")
    if len(pieces) > 2 or not all(p.strip() for p in pieces):
        raise ValueError(f"{where}: cannot read threshold {text!r} (expected 'upper' or 'lower_upper')")
    try:
        nums = [float(p) for p in pieces]
    except ValueError:
        raise ValueError(f"{where}: threshold {text!r} is not numeric") from None
    lower, upper = (None, nums[0]) if len(nums) == 1 else (nums[0], nums[1])
    if upper <= 0 or (lower is not None and not 0 < lower <= upper):
        raise ValueError(f"{where}: threshold {text!r} needs positive bounds with lower <= upper")
    return lower, upper


def _as_text(spec, where: str) -> str:
    if isinstance(spec, bool) or not isinstance(spec, (int, float, str)):
        raise TypeError(f"{where}: threshold must be a number or a string, got {type(spec).__name__}")
    text = str(spec).strip()
    if not text:
        raise ValueError(f"{where}: empty threshold")
    return text


def parse_is_threshold(spec) -> tuple[float, Optional[float]]:
    """``rollout_is_threshold`` -> (upper, lower or None); a band is IcePop."""
    lower, upper = _read_bound(_as_text(spec, "rollout_is_threshold"), "rollout_is_threshold")
    return upper, lower


def parse_rs_thresholds(options: list[str], spec) -> dict[str, tuple[Optional[float], float]]:
    """``rollout_rs_threshold`` (one value for all criteria, or one per
    criterion, comma separated) -> {criterion: (lower or None, upper)}."""
    if spec is None:
        raise ValueError("rejection sampling is on but rollout_rs_threshold is not set")
    tokens = [t.strip() for t in _as_text(spec, "rollout_rs_threshold").split(",") if t.strip()]
    if len(tokens) == 1:
        tokens = tokens * len(options)
    if len(tokens) != len(options):
        raise ValueError(f"rollout_rs_threshold: {len(options)} criteria need 1 or {len(options)} thresholds, "
                         f"{len(tokens)} given")
    bands: dict[str, tuple[Optional[float], float]] = {}
    for crit, tok in zip(options, tokens):
        lower, upper = _read_bound(tok, f"rollout_rs '{crit}'")
        if crit.endswith("k1"):
            bands[crit] = (1.0 / upper if lower is None else lower, upper)
        elif lower is not None:
            raise ValueError(f"rollout_rs '{crit}': only an upper bound applies, got band {tok!r}")
        else:
            bands[crit] = (None, upper)
    return bands


# ---------------------------------------------------------------------------
# rejection sampling
# ---------------------------------------------------------------------------

def compute_rollout_rejection_mask(log_ratio: Tensor, response_mask: Tensor, rollout_rs: str = "token_k1",
                                   rollout_rs_threshold=None) -> tuple[Tensor, dict[str, float]]:
    if not isinstance(rollout_rs, str) or not rollout_rs:
        raise ValueError("rollout_rs must be a non-empty string.")
    if rollout_rs_threshold is None:
        raise ValueError("rollout_rs_threshold must be provided.")
    if log_ratio.shape[0] == 0:
        return response_mask, {}
    opts: list[str] = []
    for o in (x.strip() for x in rollout_rs.split(",")):
        if not o:
            continue
        if o not in SUPPORTED_ROLLOUT_RS_OPTIONS:
            raise ValueError(f"Invalid rollout_rs option: {o}. Must be one of {sorted(SUPPORTED_ROLLOUT_RS_OPTIONS)}.")
        if o not in opts:
            opts.append(o)
    if not opts:
        raise ValueError("rollout_rs must contain at least one option.")
    th = parse_rs_thresholds(opts, rollout_rs_threshold)

    lr = log_ratio.clamp(-SAFETY_BOUND, SAFETY_BOUND)
    stats = {"k1": -lr, "k2": 0.5 * lr * lr, "k3": torch.exp(lr) - 1.0 - lr}
    mb = response_mask.bool()
    keep_all = torch.ones_like(response_mask, dtype=log_ratio.dtype)
    metrics: dict[str, float] = {}
    for opt in opts:
        lo, hi = th[opt]
        kind = opt[-2:]
        tok = stats[kind]
        if opt.startswith("token"):
            val = tok
        elif opt.startswith("seq_sum"):
            val = _msum(tok, response_mask, -1).unsqueeze(-1)
        elif opt.startswith("seq_mean"):
            val = _mmean(tok, response_mask, -1).unsqueeze(-1)
        else:  # seq_max
            mx = tok.masked_fill(~mb, float("-inf")).max(-1).values
            val = torch.where(torch.isinf(mx), torch.zeros_like(mx), mx).unsqueeze(-1)
        if kind == "k1":
            keep = (val >= math.log(lo)) & (val <= math.log(hi))
        else:
            keep = val <= hi
        keep = keep.expand_as(mb)
        kf = keep.to(log_ratio.dtype)
        keep_all = keep_all * kf
        metrics[f"rollout_rs_{opt}_masked_fraction"] = _mmean(1.0 - kf, response_mask).item()
        valid = mb.any(-1)
        seq_kept = (keep | ~mb).all(-1)
        metrics[f"rollout_rs_{opt}_seq_masked_fraction"] = (
            ((~seq_kept) & valid).float().sum() / valid.float().sum()).item() if bool(valid.any()) else 0.0
    metrics["rollout_rs_masked_fraction"] = _mmean(1.0 - keep_all, response_mask).item()
    final = (keep_all > 0.5) & mb
    metrics["rollout_rs_seq_masked_fraction"] = ((~final) & mb).any(-1).float().mean().item()
    return (response_mask * keep_all).to(response_mask.dtype), metrics


# ---------------------------------------------------------------------------
# importance weights
# ---------------------------------------------------------------------------

def _seq_log_ratio(log_ratio: Tensor, mask: Tensor, reduction: str = "sum") -> Tensor:
    s = _msum(log_ratio, mask, -1).unsqueeze(-1)
    if reduction == "mean":
        return s / mask.sum(-1, keepdim=True).clamp(min=1).to(s.dtype)
    return s


def compute_rollout_correction_weights(log_ratio: Tensor, response_mask: Tensor, rollout_is: str = "token",
                                       rollout_is_threshold=2.0, rollout_is_batch_normalize: bool = False,
                                       rollout_is_seq_reduction: str = "sum") -> tuple[Tensor, dict[str, float]]:
    if rollout_is not in ("token", "sequence"):
        raise ValueError(f"Invalid rollout_is: {rollout_is}. Must be one of {{'token', 'sequence'}}.")
    upper, lower = parse_is_threshold(rollout_is_threshold)
    icepop = lower is not None
    lower_eff = lower if icepop else 1.0 / upper
    if rollout_is == "token":
        raw = torch.exp(log_ratio.clamp(-SAFETY_BOUND, SAFETY_BOUND))
    else:
        seq_lr = _seq_log_ratio(log_ratio, response_mask, rollout_is_seq_reduction)
        raw = torch.exp(seq_lr.clamp(-SAFETY_BOUND, SAFETY_BOUND)).expand_as(log_ratio)
    raw = raw * response_mask
    if icepop:
        w = torch.where((raw >= lower) & (raw <= upper), raw, torch.zeros_like(raw))
    else:
        w = raw.clamp(max=upper)

    mb = response_mask.bool()
    m: dict[str, float] = {"rollout_is_mean": _mmean(w, response_mask).item()}
    if rollout_is == "token":
        m["rollout_is_ratio_fraction_high"] = _mmean((raw > upper).float(), response_mask).item()
        m["rollout_is_ratio_fraction_low"] = _mmean((raw < lower_eff).float(), response_mask).item()
        m["rollout_is_max"] = w.masked_fill(~mb, float("-inf")).max().item()
        m["rollout_is_min"] = w.masked_fill(~mb, float("inf")).min().item()
    else:
        s = _seq_log_ratio(log_ratio, response_mask, rollout_is_seq_reduction)
        m["rollout_is_max"] = math.exp(min(s.max().item(), SAFETY_BOUND))
        m["rollout_is_min"] = math.exp(s.min().item())
        m["rollout_is_ratio_fraction_high"] = (s > math.log(upper)).float().mean().item()
        m["rollout_is_ratio_fraction_low"] = (s < math.log(lower_eff)).float().mean().item()
    wc = w.clamp(0.0, upper)
    if response_mask.sum() > 1:
        mu = _mmean(wc, response_mask)
        m["rollout_is_std"] = torch.sqrt((_mmean(wc * wc, response_mask) - mu * mu).clamp(min=0)).item()
    else:
        m["rollout_is_std"] = 0.0
    wn = wc / (_mmean(wc, response_mask) + 1e-8)
    m["rollout_is_eff_sample_size"] = 1.0 / _mmean(wn * wn, response_mask).item()
    if w.dim() > 1:
        sm = _mmean(w, response_mask, -1)
        m["rollout_is_seq_mean"] = sm.mean().item()
        m["rollout_is_seq_std"] = sm.std().item() if sm.numel() > 1 else 0.0
        m["rollout_is_seq_max"] = sm.max().item()
        m["rollout_is_seq_min"] = sm.min().item()
        m["rollout_is_seq_max_deviation"] = (sm - 1.0).abs().max().item()
        rsm = _mmean(raw, response_mask, -1)
        m["rollout_is_seq_fraction_high"] = (rsm > upper).float().mean().item()
        m["rollout_is_seq_fraction_low"] = (rsm < lower_eff).float().mean().item()
    if icepop:
        m["rollout_is_oob_ratio"] = _mmean(((raw < lower) | (raw > upper)).float(), response_mask).item()
    w = w.detach()
    if rollout_is_batch_normalize:
        if rollout_is == "token":
            mu = _mmean(w, response_mask)
        else:
            seq_w = _mmean(w, response_mask, -1)
            seq_m = (response_mask.sum(-1) > 0).to(w.dtype)
            mu = (seq_w * seq_m).sum() / seq_m.sum().clamp(min=1e-8)
        if mu > 1e-8:
            w = w / mu
            m["rollout_is_batch_norm_factor"] = mu.item()
        else:
            m["rollout_is_batch_norm_factor"] = 1.0
    return w, m


def compute_offpolicy_metrics(old_log_prob: Tensor, rollout_log_prob: Optional[Tensor],
                              response_mask: Tensor) -> dict[str, Any]:
    """Perplexities and train/rollout divergences, all read back to the host
    in one transfer."""
    lp_train = _mmean(old_log_prob, response_mask, -1)
    vals: dict[str, Tensor] = {"training_ppl": torch.exp(-lp_train).mean(), "training_log_ppl": (-lp_train).mean()}
    if rollout_log_prob is not None:
        lr = old_log_prob - rollout_log_prob
        lp_roll = _mmean(rollout_log_prob, response_mask, -1)
        d = lp_roll - lp_train
        rho = torch.exp(lr.clamp(-SAFETY_BOUND, SAFETY_BOUND))
        s = _msum(lr, response_mask, -1).clamp(-SAFETY_BOUND, SAFETY_BOUND)
        vals.update({
            "kl": _mmean(-lr, response_mask),
            "k3_kl": _mmean(torch.exp(lr) - lr - 1, response_mask),
            "rollout_ppl": torch.exp(-lp_roll).mean(), "rollout_log_ppl": (-lp_roll).mean(),
            "log_ppl_diff": d.mean(), "log_ppl_abs_diff": d.abs().mean(),
            "log_ppl_diff_max": d.max(), "log_ppl_diff_min": d.min(),
            "ppl_ratio": torch.exp(d).mean(),
            "chi2_token": _mmean(rho * rho, response_mask) - 1.0,
            "chi2_seq": torch.exp(2.0 * s).mean() - 1.0,
        })
    host = torch.stack([v.reshape(()).float() for v in vals.values()]).cpu().tolist()
    return dict(zip(vals.keys(), host))


# train/rollout mismatch beyond the signed mean (reference:
# ``workers/actor_worker.py:760-792``, ``trainer/rl_trainer.py:3630-3652``):
# per-rank SUMS with their denominators, so a cross-rank sum gives exact
# token- and sequence-weighted means
MISMATCH_TOKEN_KEYS = ("mismatch/abs_diff", "mismatch/k3_kl", "mismatch/chi2_token", "mismatch/frac_abs_gt_0.1")


def mismatch_sums(train_log_prob: Tensor, rollout_log_prob: Tensor, response_mask: Tensor) -> Tensor:
    """[sum |r|, sum (e^r - 1 - r), sum (e^r - 1)^2, count |r| > 0.1, tokens,
    sum over rows (e^{sum r} - 1)^2, rows] on the device, r = train - rollout
    log-prob per response token (clamped to +-10 inside the exponentials)."""
    mask = response_mask.to(train_log_prob.dtype)
    r = (train_log_prob - rollout_log_prob) * mask
    w = torch.exp(r.clamp(-10.0, 10.0))
    w_seq = torch.exp(r.sum(-1).clamp(-10.0, 10.0))
    return torch.stack([r.abs().sum(), ((w - 1.0 - r) * mask).sum(), ((w - 1.0) ** 2 * mask).sum(),
                        ((r.abs() > 0.1).to(r.dtype) * mask).sum(), mask.sum(), ((w_seq - 1.0) ** 2).sum(),
                        torch.tensor(float(r.shape[0]), dtype=r.dtype, device=r.device)]).double()


def finalize_mismatch(sums) -> dict[str, float]:
    """Means from (cross-rank summed) ``mismatch_sums``."""
    a, k3, c2, tail, tok, c2s, rows = (float(x) for x in sums)
    out = {k: v / max(tok, 1e-6) for k, v in zip(MISMATCH_TOKEN_KEYS, (a, k3, c2, tail))} if tok else {}
    if rows:
        out["mismatch/chi2_seq"] = c2s / max(rows, 1e-6)
    return out


_LEGACY_ALIASES = {"is_weight_mean": "rollout_is_mean", "is_weight_max": "rollout_is_max", "kl": "kl", "k3_kl": "k3_kl"}


def compute_rollout_correction_and_rejection_mask(old_log_prob: Tensor, rollout_log_prob: Tensor,
                                                  response_mask: Tensor, rollout_is: Optional[str] = None,
                                                  rollout_is_threshold=2.0, rollout_is_batch_normalize: bool = False,
                                                  rollout_rs: Optional[str] = None, rollout_rs_threshold=None,
                                                  rollout_is_seq_reduction: str = "sum"):
    lr = old_log_prob - rollout_log_prob
    metrics: dict[str, float] = {}
    w = None
    if rollout_is is not None and rollout_is_threshold is not None:
        w, mm = compute_rollout_correction_weights(lr, response_mask, rollout_is, rollout_is_threshold,
                                                   rollout_is_batch_normalize, rollout_is_seq_reduction)
        metrics.update(mm)
    new_mask = response_mask.clone()
    if rollout_rs is not None:
        if rollout_rs_threshold is None:
            raise ValueError("rollout_rs_threshold must be provided when rollout_rs is enabled.")
        new_mask, mm = compute_rollout_rejection_mask(lr, response_mask, rollout_rs, rollout_rs_threshold)
        metrics.update(mm)
    metrics.update(compute_offpolicy_metrics(old_log_prob, rollout_log_prob, response_mask))
    out = {f"rollout_corr/{k}": float(v) for k, v in metrics.items()}
    for legacy, new in _LEGACY_ALIASES.items():
        if new in metrics:
            out[f"rollout_correction/{legacy}"] = float(metrics[new])
    return w, new_mask, out


def _resolve_cfg(config: Any) -> RolloutCorrectionConfig:
    if isinstance(config, RolloutCorrectionConfig):
        return config
    if isinstance(config, QuantizationConfig):
        return config.rollout_correction
    if isinstance(config, LumenRLConfig):
        return config.quantization.rollout_correction
    raise TypeError(f"Expected RolloutCorrectionConfig, got {type(config)!r}")


def _aligned_logprobs(batch: DataProto) -> tuple[Tensor, Tensor, Tensor, str]:
    """Trim old/rollout/mask to a common width and de-alias unreported zeros."""
    old = batch.tensors["old_log_probs"]
    roll = batch.tensors.get("rollout_log_probs", batch.tensors.get("fp8_logprobs"))
    mkey = "response_mask" if "response_mask" in batch.tensors else "attention_mask"
    mask = batch.tensors.get(mkey)
    if roll is None or mask is None:
        raise KeyError("rollout correction needs rollout_log_probs (or fp8_logprobs) and "
                       "response_mask (or attention_mask) in the batch")
    w = min(old.shape[-1], roll.shape[-1], mask.shape[-1])
    o, r, m = old[..., :w], roll[..., :w], mask[..., :w]
    holes = (r == 0.0) & (m > 0)
    if bool(holes.any()):
        r = torch.where(holes, o, r)
        patched = roll.clone()
        patched[..., :w] = r
        batch.tensors["rollout_log_probs"] = patched
        logger.info("rollout_log_probs: %d response positions were exactly 0.0; used old_log_probs there",
                    int(holes.sum()))
    return o, r, m, mkey


def compute_rollout_correction_and_add_to_batch(batch: DataProto, config: Any) -> tuple[DataProto, dict[str, float]]:
    c = _resolve_cfg(config)
    o, r, m, mkey = _aligned_logprobs(batch)
    w, new_mask, metrics = compute_rollout_correction_and_rejection_mask(
        o, r, m, rollout_is=c.rollout_is or None, rollout_is_threshold=c.rollout_is_threshold or None,
        rollout_is_batch_normalize=c.rollout_is_batch_normalize, rollout_rs=c.rollout_rs or None,
        rollout_rs_threshold=c.rollout_rs_threshold or None, rollout_is_seq_reduction=c.rollout_is_seq_reduction)
    orig = batch.tensors[mkey]
    if new_mask.shape[-1] == orig.shape[-1]:
        batch.tensors[mkey] = new_mask
    else:
        full = orig.clone()
        full[..., : new_mask.shape[-1]] = new_mask
        batch.tensors[mkey] = full
    if w is not None:
        batch.tensors["rollout_is_weights"] = w
    return batch, metrics


def compute_rollout_corr_metrics_from_logprobs(log_prob: Tensor, rollout_log_prob: Tensor,
                                               response_mask: Tensor) -> dict[str, float]:
    return {f"rollout_corr/{k}": float(v) for k, v in
            compute_offpolicy_metrics(log_prob, rollout_log_prob, response_mask).items()}


def apply_bypass_mode(batch: DataProto, config: Any) -> None:
    if "rollout_log_probs" not in batch.tensors:
        raise ValueError("bypass_mode=True requires rollout_log_probs in batch. "
                         "Ensure calculate_log_probs=true in rollout config.")
    batch.tensors["old_log_probs"] = batch.tensors["rollout_log_probs"]


# ---- legacy advantage-level corrections -----------------------------------

def token_level_tis(bf16_logprobs: Tensor, fp8_logprobs: Tensor, advantages: Tensor, clip: float = 1.5) -> Tensor:
    ratio = torch.exp((bf16_logprobs - fp8_logprobs).clamp(-20.0, 20.0))
    return ratio.clamp(1.0 / clip, clip) * advantages


def token_level_mis(bf16_logprobs: Tensor, fp8_logprobs: Tensor, advantages: Tensor) -> Tensor:
    ratio = torch.exp((bf16_logprobs - fp8_logprobs).clamp(-20.0, 20.0))
    return ratio / ratio.mean().clamp(min=1e-8) * advantages


def _first_key(batch: DataProto, keys: tuple[str, ...], what: str) -> Tensor:
    for k in keys:
        if k in batch.tensors:
            return batch.tensors[k]
    raise KeyError(f"DataProto must contain one of {keys} ({what}).")


def apply_rollout_correction(batch: DataProto, config: Any) -> DataProto:
    c = _resolve_cfg(config)
    if not c.enabled:
        return batch
    hi = _first_key(batch, ("bf16_logprobs", "old_log_probs", "ref_log_probs"), "high-precision log-probs")
    lo = _first_key(batch, ("fp8_logprobs", "fp8_log_probs"), "rollout log-probs")
    if "advantages" not in batch.tensors:
        raise KeyError("DataProto must contain 'advantages' for rollout correction.")
    method = c.method.lower().strip()
    if method == "tis":
        adv = token_level_tis(hi, lo, batch["advantages"], clip=c.clip)
    elif method in ("mis", "multiplicative"):
        adv = token_level_mis(hi, lo, batch["advantages"])
    else:
        raise ValueError(f"Unknown rollout correction method: {c.method!r}")
    out = DataProto(dict(batch.tensors), dict(batch.meta), batch.ragged)
    out["advantages"] = adv
    out.meta["rollout_correction"] = {"method": method, "clip": c.clip}
    return out


def compute_rollout_is_weights(old_log_probs: Tensor, rollout_log_probs: Tensor, response_mask: Tensor,
                               rollout_is: str = "token", rollout_is_threshold=2.0,
                               rollout_is_batch_normalize: bool = False):
    w, m = compute_rollout_correction_weights(old_log_probs - rollout_log_probs, response_mask, rollout_is,
                                              rollout_is_threshold, rollout_is_batch_normalize)
    return w * response_mask, {f"rollout_correction/{k}": v for k, v in m.items()}


def apply_rejection_sampling(response_mask: Tensor, is_weights: Tensor, threshold: float = 0.0) -> Tensor:
    if threshold <= 0.0:
        return response_mask
    out = response_mask.clone()
    out[is_weights > threshold] = 0
    return out


# ---- presets ----------------------------------------------------------------

def _rc(**kw) -> RolloutCorrectionConfig:
    return RolloutCorrectionConfig(**kw)


def preset_decoupled_token_is(threshold: float = 2.0):
    return _rc(rollout_is="token", rollout_is_threshold=str(threshold))


def preset_decoupled_seq_is(threshold: float = 2.0):
    return _rc(rollout_is="sequence", rollout_is_threshold=str(threshold))


def preset_decoupled_token_icepop(lower: float = 0.5, upper: float = 5.0):
    return _rc(rollout_is="token", rollout_is_threshold=f"{lower}_{upper}")


def preset_decoupled_seq_is_rs(is_threshold: float = 2.0, rs_threshold: str = "0.5_2.0"):
    return _rc(rollout_is="sequence", rollout_is_threshold=str(is_threshold),
               rollout_rs="seq_sum_k1", rollout_rs_threshold=rs_threshold)


def preset_decoupled_geo_rs(threshold: str = "0.999_1.001"):
    return _rc(rollout_rs="seq_mean_k1", rollout_rs_threshold=threshold)


def preset_decoupled_geo_rs_seq_tis(is_threshold: float = 2.0, rs_threshold: str = "0.999_1.001"):
    return _rc(rollout_is="sequence", rollout_is_threshold=str(is_threshold),
               rollout_rs="seq_mean_k1", rollout_rs_threshold=rs_threshold)


def preset_decoupled_geo_rs_token_tis(is_threshold: float = 2.0, rs_threshold: str = "0.999_1.001"):
    return _rc(rollout_is="token", rollout_is_threshold=str(is_threshold),
               rollout_rs="seq_mean_k1", rollout_rs_threshold=rs_threshold)


def preset_decoupled_k3_rs(threshold: float = 0.005):
    return _rc(rollout_rs="seq_mean_k3", rollout_rs_threshold=str(threshold))


def preset_decoupled_k3_rs_seq_tis(is_threshold: float = 2.0, rs_threshold: float = 0.005):
    return _rc(rollout_is="sequence", rollout_is_threshold=str(is_threshold),
               rollout_rs="seq_mean_k3", rollout_rs_threshold=str(rs_threshold))


def preset_decoupled_k3_rs_token_tis(is_threshold: float = 2.0, rs_threshold: float = 0.005):
    return _rc(rollout_is="token", rollout_is_threshold=str(is_threshold),
               rollout_rs="seq_mean_k3", rollout_rs_threshold=str(rs_threshold))


def preset_bypass_ppo_clip():
    return _rc(bypass_mode=True, loss_type="ppo_clip")


def preset_bypass_ppo_clip_geo_rs(rs_threshold: str = "0.999_1.001"):
    return _rc(bypass_mode=True, loss_type="ppo_clip", rollout_rs="seq_mean_k1", rollout_rs_threshold=rs_threshold)


def preset_bypass_ppo_clip_k3_rs(rs_threshold: float = 0.005):
    return _rc(bypass_mode=True, loss_type="ppo_clip", rollout_rs="seq_mean_k3",
               rollout_rs_threshold=str(rs_threshold))


def preset_bypass_pg_is(threshold: float = 2.0):
    return _rc(bypass_mode=True, loss_type="reinforce", rollout_is="sequence", rollout_is_threshold=str(threshold))


def preset_bypass_pg_geo_rs(rs_threshold: str = "0.999_1.001"):
    return _rc(bypass_mode=True, loss_type="reinforce", rollout_rs="seq_mean_k1", rollout_rs_threshold=rs_threshold)


def preset_bypass_pg_geo_rs_seq_tis(is_threshold: float = 2.0, rs_threshold: str = "0.999_1.001"):
    return _rc(bypass_mode=True, loss_type="reinforce", rollout_is="sequence", rollout_is_threshold=str(is_threshold),
               rollout_rs="seq_mean_k1", rollout_rs_threshold=rs_threshold)


def preset_bypass_pg_geo_rs_token_tis(is_threshold: float = 2.0, rs_threshold: str = "0.999_1.001"):
    return _rc(bypass_mode=True, loss_type="reinforce", rollout_is="token", rollout_is_threshold=str(is_threshold),
               rollout_rs="seq_mean_k1", rollout_rs_threshold=rs_threshold)


def preset_disabled():
    return _rc()
