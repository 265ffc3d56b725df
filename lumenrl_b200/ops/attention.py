"""Packed (varlen) causal attention for training and prefill.

``flash_attention_varlen`` runs the sequences of a packed batch through
PyTorch's fused SDPA (one call per sequence, GQA native).  The hand-written
tcgen05 kernel (``csrc/attn/fa_varlen``) replaces this when built; until then
this path is the library baseline for the attention share of the step.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import Tensor


def flash_attention_varlen(q: Tensor, k: Tensor, v: Tensor, cu_seqlens: Tensor, max_seqlen: int,
                           causal: bool = True, scale: float | None = None) -> Tensor:
    cu = cu_seqlens.tolist()
    outs = []
    for i in range(len(cu) - 1):
        a, b = cu[i], cu[i + 1]
        if b <= a:
            continue
        qi = q[a:b].transpose(0, 1).unsqueeze(0)
        ki = k[a:b].transpose(0, 1).unsqueeze(0)
        vi = v[a:b].transpose(0, 1).unsqueeze(0)
        o = F.scaled_dot_product_attention(qi, ki, vi, is_causal=causal, scale=scale, enable_gqa=True)
        outs.append(o.squeeze(0).transpose(0, 1))
    return torch.cat(outs, 0) if len(outs) > 1 else outs[0].contiguous()
