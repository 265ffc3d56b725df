"""Ulysses sequence parallelism (reference ``utils/ulysses.py:102-346``,
defined there but unused by its engines).

Activations are sharded by sequence across the group of ``P`` ranks.  Around
attention an all-to-all turns ``[T/P, H, D]`` sequence shards into
``[T, H/P, D]`` head shards (every rank then sees whole sequences for its
heads, so causal attention needs no ring), and a second all-to-all turns the
output back.  Both are differentiable (the backward of one all-to-all is the
inverse all-to-all).  Heads (and KV heads) must divide by ``P``.
"""

from __future__ import annotations

import torch
import torch.distributed as dist
from torch import Tensor


def _a2a(x: Tensor, group, scatter_dim: int, gather_dim: int) -> Tensor:
    P = dist.get_world_size(group)
    if P == 1:
        return x
    send = torch.stack(x.chunk(P, dim=scatter_dim)).contiguous()   # [P, chunk...]
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)                # equal splits along dim 0
    return torch.cat(list(recv.unbind(0)), dim=gather_dim)


class _SeqToHead(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return _a2a(x, group, scatter_dim=1, gather_dim=0)

    @staticmethod
    def backward(ctx, g):
        return _a2a(g, ctx.group, scatter_dim=0, gather_dim=1), None


class _HeadToSeq(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return _a2a(x, group, scatter_dim=0, gather_dim=1)

    @staticmethod
    def backward(ctx, g):
        return _a2a(g, ctx.group, scatter_dim=1, gather_dim=0), None


def seq_to_head(x: Tensor, group=None) -> Tensor:
    """[T/P, H, D] (this rank's tokens, all heads) -> [T, H/P, D]."""
    return _SeqToHead.apply(x, group)


def head_to_seq(x: Tensor, group=None) -> Tensor:
    """[T, H/P, D] (all tokens, this rank's heads) -> [T/P, H, D]."""
    return _HeadToSeq.apply(x, group)


def ulysses_attention(q: Tensor, k: Tensor, v: Tensor, cu_seqlens: Tensor, max_seqlen: int, group=None,
                      scale=None) -> Tensor:
    """Causal packed attention on sequence-sharded q [T/P, Hq, D], k/v
    [T/P, Hk, D]; ``cu_seqlens`` describes the FULL packed batch."""
    from lumenrl_b200 import ops
    qh, kh, vh = seq_to_head(q, group), seq_to_head(k, group), seq_to_head(v, group)
    o = ops.attention_varlen(qh, kh, vh, cu_seqlens, max_seqlen, causal=True, scale=scale)
    return head_to_seq(o, group)
