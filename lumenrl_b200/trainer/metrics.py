"""Metric naming and cross-rank reduction (reference
``lumenrl/trainer/metric_utils.py:22-224``, ``rl_trainer.py:3480-3506``).

* ``reduce_metrics``: keys ending in ``/max`` reduce with MAX, ``/min`` with
  MIN, everything else with the mean over ranks; ``*_sum``/``*_tok`` pairs
  reduce with SUM so token-weighted means stay exact.
* ``throughput_metrics``: ``perf/throughput = tokens / (step_time * n_gpus)``
  (the reference formula), ``perf/step_tokens_per_s`` = whole-job tokens/s.
* verl-style aliases for dashboards.
"""

from __future__ import annotations

from typing import Mapping

import torch
import torch.distributed as dist

VERL_ALIASES = {"actor/pg_loss": "actor/pg_loss", "actor/pg_clipfrac": "actor/pg_clipfrac",
                "actor/ppo_kl": "actor/ppo_kl", "actor/entropy": "actor/entropy", "reward/mean": "critic/score/mean",
                "response_length/mean": "response_length/mean", "timing/step_s": "timing_s/step",
                "timing/gen_s": "timing_s/gen", "timing/train_s": "timing_s/update_actor",
                "timing/old_log_prob_s": "timing_s/old_log_prob"}


def reduce_metrics(m: Mapping[str, float], device="cpu") -> dict[str, float]:
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return dict(m)
    w = dist.get_world_size()
    keys = sorted(k for k, v in m.items() if isinstance(v, (int, float)))
    out = {}
    groups = {"max": [], "min": [], "sum": [], "mean": []}
    for k in keys:
        if k.endswith("/max"):
            groups["max"].append(k)
        elif k.endswith("/min"):
            groups["min"].append(k)
        elif k.endswith("_sum") or k.endswith("_tok"):
            groups["sum"].append(k)
        else:
            groups["mean"].append(k)
    for kind, ks in groups.items():
        if not ks:
            continue
        t = torch.tensor([float(m[k]) for k in ks], dtype=torch.float64, device=device)
        op = {"max": dist.ReduceOp.MAX, "min": dist.ReduceOp.MIN}.get(kind, dist.ReduceOp.SUM)
        dist.all_reduce(t, op=op)
        if kind == "mean":
            t /= w
        out.update(dict(zip(ks, t.tolist())))
    return out


def throughput_metrics(total_tokens: float, step_s: float, n_gpus: int) -> dict[str, float]:
    return {"perf/total_num_tokens": total_tokens, "perf/time_per_step": step_s,
            "perf/throughput": total_tokens / max(step_s * n_gpus, 1e-9),
            "perf/step_tokens_per_s": total_tokens / max(step_s, 1e-9)}


def with_aliases(m: Mapping[str, float]) -> dict[str, float]:
    out = dict(m)
    for k, a in VERL_ALIASES.items():
        if k in m and a not in out:
            out[a] = m[k]
    return out
