"""DAPO sampling helpers (reference ``lumenrl/algorithms/dapo_sampling.py:30-106``).

* ``overlong_buffer_penalty``: soft penalty that is 0 up to
  ``max_resp_len - buffer_len`` tokens and falls linearly by
  ``penalty_factor`` over the last ``buffer_len`` tokens (and beyond).
* ``filter_groups_keep_mask``: dynamic sampling -- drop prompt groups whose
  metric has zero (population) std; singleton groups are kept.
"""

from __future__ import annotations

from typing import Sequence

import torch
from torch import Tensor


def overlong_buffer_penalty(response_lengths, max_resp_len: int, buffer_len: int,
                            penalty_factor: float) -> Tensor:
    lens = torch.as_tensor(response_lengths, dtype=torch.float32)
    if buffer_len <= 0 or penalty_factor == 0.0:
        return torch.zeros_like(lens)
    excess = lens - float(max_resp_len - buffer_len)
    return (-excess / float(buffer_len) * float(penalty_factor)).clamp(max=0.0)


def filter_groups_keep_mask(metric_vals, uids: Sequence, *, eps: float = 0.0) -> tuple[Tensor, list]:
    vals = torch.as_tensor(metric_vals, dtype=torch.float32).reshape(-1)
    if len(uids) != vals.shape[0]:
        raise ValueError(f"len(uids)={len(uids)} != metric_vals={vals.shape[0]}")
    order: dict = {}
    for u in uids:
        order.setdefault(u, len(order))
    gid = torch.as_tensor([order[u] for u in uids], dtype=torch.long)
    ng = len(order)
    cnt = torch.zeros(ng).index_add_(0, gid, torch.ones_like(vals))
    mean = torch.zeros(ng).index_add_(0, gid, vals) / cnt
    var = torch.zeros(ng).index_add_(0, gid, (vals - mean[gid]) ** 2) / cnt
    keep_group = (cnt == 1) | (var.sqrt() > eps)
    kept = [u for u, i in order.items() if bool(keep_group[i])]
    return keep_group[gid].clone(), kept
