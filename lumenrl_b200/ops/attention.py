"""Packed (varlen) causal attention for training and prefill.

``flash_attention_varlen`` runs the whole packed batch in one call of the
flash-attention varlen kernel that ships with PyTorch
(``aten._flash_attention_forward`` / ``_backward``: cumulative sequence
lengths, native GQA, log-sum-exp kept for the backward).  No per-sequence
loop and no device->host read of ``cu_seqlens``: ``max_seqlen`` comes from the
caller, who packed the batch on the host.  This is the library attention of
the training step (the reference also calls a library kernel here,
``engine/training/packing.py:363-421``).

By default (bf16, head dim 128, causal) both directions run on this
package's tcgen05 kernels: the forward ``csrc/attn/fa_fwd.cu`` writes the
log-sum-exp in the varlen layout ``[Hq, T]``, the backward
``csrc/attn/fa_bwd.cu`` reads it.  ``LRL_TRAIN_ATTN_BWD=fa2`` feeds that
output and LSE to the library backward instead; ``LRL_TRAIN_ATTN=fa2`` puts
both directions on the library kernels.
"""

from __future__ import annotations

import os

import torch
import torch.nn.functional as F
from torch import Tensor

TRAIN_ATTN = os.environ.get("LRL_TRAIN_ATTN", "tc")    # "tc" (own tcgen05 forward) | "fa2" (library)
TRAIN_ATTN_BWD = os.environ.get("LRL_TRAIN_ATTN_BWD", "tc")    # backward after the tcgen05 forward: "tc" | "fa2"


class _VarlenFlash(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, cu, max_len, causal, scale):
        q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
        out, lse, seed, offset, _ = torch.ops.aten._flash_attention_forward(
            q, k, v, cu, cu, max_len, max_len, 0.0, causal, False, scale=scale)
        ctx.save_for_backward(q, k, v, out, lse, cu, seed, offset)
        ctx.max_len, ctx.causal, ctx.scale = max_len, causal, scale
        return out

    @staticmethod
    def backward(ctx, do):
        q, k, v, out, lse, cu, seed, offset = ctx.saved_tensors
        dq, dk, dv = torch.ops.aten._flash_attention_backward(
            do.contiguous(), q, k, v, out, lse, cu, cu, ctx.max_len, ctx.max_len, 0.0, ctx.causal, seed, offset,
            scale=ctx.scale)
        return dq, dk, dv, None, None, None, None


class _VarlenTC(torch.autograd.Function):
    """Forward on the tcgen05 kernel, backward on the library kernel (fed
    the forward's output and LSE; no dropout, so no RNG state)."""

    @staticmethod
    def forward(ctx, q, k, v, cu, max_len, scale):
        from lumenrl_b200.ops.ext import ext
        q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
        out, lse = ext().fa_fwd(q, k, v, cu, max_len, scale)
        ctx.save_for_backward(q, k, v, out, lse, cu)
        ctx.max_len, ctx.scale = max_len, scale
        return out

    @staticmethod
    def backward(ctx, do):
        q, k, v, out, lse, cu = ctx.saved_tensors
        if TRAIN_ATTN_BWD == "tc":
            from lumenrl_b200.ops.ext import ext
            dq, dk, dv = ext().fa_bwd(do.contiguous(), q, k, v, out, lse, cu, ctx.max_len, ctx.scale)
            return dq, dk, dv, None, None, None
        zero = torch.zeros((), dtype=torch.int64, device=q.device)
        dq, dk, dv = torch.ops.aten._flash_attention_backward(
            do.contiguous(), q, k, v, out, lse, cu, cu, ctx.max_len, ctx.max_len, 0.0, True, zero, zero,
            scale=ctx.scale)
        return dq, dk, dv, None, None, None


def tc_attention_ok(q: Tensor, causal: bool) -> bool:
    return causal and q.is_cuda and q.dtype == torch.bfloat16 and q.shape[-1] == 128


def flash_attention_varlen(q: Tensor, k: Tensor, v: Tensor, cu_seqlens: Tensor, max_seqlen: int,
                           causal: bool = True, scale: float | None = None) -> Tensor:
    """q [T, Hq, D], k/v [T, Hk, D] (bf16/fp16, CUDA) packed by ``cu_seqlens``."""
    if scale is None:
        scale = q.shape[-1] ** -0.5
    cu = cu_seqlens.to(torch.int32)
    if TRAIN_ATTN == "tc" and tc_attention_ok(q, causal):
        return _VarlenTC.apply(q, k, v, cu, int(max_seqlen), float(scale))
    if q.dtype in (torch.bfloat16, torch.float16):
        return _VarlenFlash.apply(q, k, v, cu, int(max_seqlen), causal, float(scale))
    # fp32 fallback: per-sequence SDPA
    bounds = cu.tolist()
    outs = []
    for a, b in zip(bounds[:-1], bounds[1:]):
        if b > a:
            o = F.scaled_dot_product_attention(q[a:b].transpose(0, 1)[None], k[a:b].transpose(0, 1)[None],
                                               v[a:b].transpose(0, 1)[None], is_causal=causal, scale=scale,
                                               enable_gqa=True)
            outs.append(o[0].transpose(0, 1))
    return torch.cat(outs, 0)
