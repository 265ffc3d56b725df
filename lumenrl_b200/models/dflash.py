"""DFlash draft model for speculative decoding (reference
``lumenrl/models/dflash.py:31-184``).

* K teacher layers' hidden states ``[B, T, D]`` are concatenated and projected
  back to D (``layer_proj``, only when K > 1), then LayerNorm.
* ``num_layers`` pre-norm blocks: multi-head self-attention (bias on the
  in/out projections) under the block-causal mask, then a SwiGLU FFN of width
  4D (``w2(silu(w1 h) * w3 h)``).
* Final LayerNorm, logits through the frozen teacher ``lm_head``.
* Loss: cross-entropy of position t against ``target_ids[:, t+1]`` weighted by
  ``exp(-t / gamma)`` (and the loss mask), plus top-1 accuracy.

The block-causal rule (token i sees every position before its block's start
and the positions of its own block up to i) admits exactly the positions
<= i, so attention runs as causal flash attention (``is_causal``) and the
mask is never materialised.  The CE goes through the chunked LM-head
log-prob op, so ``[B, T, V]`` logits exist only when asked for.
"""

from __future__ import annotations

from typing import Optional, Union

import torch
import torch.nn as nn
import torch.nn.functional as F
from torch import Tensor

from lumenrl_b200 import ops


def block_causal_mask(seq_len: int, block_size: int, device=None) -> Tensor:
    """Boolean [T, T] mask (True = attend) of the block-causal rule, for
    inspection and tests (it equals the causal mask)."""
    i = torch.arange(seq_len, device=device)
    start = ((i // block_size) * block_size).unsqueeze(1)
    j = i.unsqueeze(0)
    return (j < start) | ((j >= start) & (j <= i.unsqueeze(1)))


class DFlashBlock(nn.Module):
    def __init__(self, dim: int, heads: int) -> None:
        super().__init__()
        self.heads = heads
        self.attn_norm = nn.LayerNorm(dim)
        self.qkv = nn.Linear(dim, 3 * dim, bias=True)
        self.out = nn.Linear(dim, dim, bias=True)
        self.ffn_norm = nn.LayerNorm(dim)
        self.w1 = nn.Linear(dim, 4 * dim, bias=False)
        self.w2 = nn.Linear(4 * dim, dim, bias=False)
        self.w3 = nn.Linear(dim, 4 * dim, bias=False)

    def forward(self, x: Tensor) -> Tensor:
        B, T, D = x.shape
        h = self.attn_norm(x)
        q, k, v = self.qkv(h).view(B, T, 3, self.heads, D // self.heads).permute(2, 0, 3, 1, 4)
        a = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        x = x + self.out(a.transpose(1, 2).reshape(B, T, D))
        h = self.ffn_norm(x)
        return x + self.w2(F.silu(self.w1(h)) * self.w3(h))


class DFlashModel(nn.Module):
    def __init__(self, hidden_dim: int, num_target_layers: int = 1, num_heads: int = 16, num_layers: int = 2,
                 block_size: int = 8) -> None:
        super().__init__()
        self.hidden_dim, self.num_target_layers, self.block_size = hidden_dim, num_target_layers, block_size
        self.layer_proj = (nn.Linear(hidden_dim * num_target_layers, hidden_dim, bias=False)
                           if num_target_layers > 1 else None)
        self.input_norm = nn.LayerNorm(hidden_dim)
        self.blocks = nn.ModuleList(DFlashBlock(hidden_dim, num_heads) for _ in range(num_layers))
        self.out_norm = nn.LayerNorm(hidden_dim)

    def hidden(self, teacher_hidden_states: Union[list, Tensor]) -> Tensor:
        x = teacher_hidden_states
        if isinstance(x, (list, tuple)):
            x = torch.cat(list(x), -1) if len(x) > 1 else x[0]
        if self.layer_proj is not None:
            x = self.layer_proj(x)
        x = self.input_norm(x)
        for blk in self.blocks:
            x = blk(x)
        return self.out_norm(x)

    def forward(self, teacher_hidden_states, lm_head_weight: Tensor, loss_mask: Optional[Tensor] = None,
                target_ids: Optional[Tensor] = None, loss_decay_gamma: float = 7.0,
                return_logits: bool = True) -> dict:
        x = self.hidden(teacher_hidden_states)
        B, T, D = x.shape
        w = lm_head_weight.detach().to(x.dtype)
        out: dict = {}
        if return_logits:
            out["logits"] = F.linear(x, w)
        if target_ids is None:
            return out
        tgt = target_ids[:, 1: T + 1]
        short = T - tgt.shape[1]
        if short > 0:
            # positions with no next token (target_ids of length T) carry no loss
            tgt = F.pad(tgt, (0, short))
            keep = torch.ones(B, T, device=x.device)
            keep[:, T - short:] = 0
            loss_mask = keep if loss_mask is None else loss_mask.to(keep.dtype) * keep
        tgt = tgt.reshape(-1)
        flat = x.reshape(-1, D)
        logp, _ = ops.token_logprob(flat, w, tgt, want_entropy=False)
        ce = -logp.view(B, T)
        decay = torch.exp(-torch.arange(T, device=x.device, dtype=torch.float32) / loss_decay_gamma)
        with torch.no_grad():
            pred = torch.cat([(c @ w.t()).argmax(-1) for c in flat.detach().split(4096)]).view(B, T)
            hit = (pred == tgt.view(B, T)).float()
        if loss_mask is not None:
            m = loss_mask.to(ce.dtype)
            wts = m * decay
            out["loss"] = (ce * wts).sum() / wts.sum().clamp(min=1.0)
            out["accuracy"] = (hit * m).sum() / m.sum().clamp(min=1.0)
        else:
            out["loss"] = (ce * decay).mean()
            out["accuracy"] = hit.mean()
        return out
