"""Vocabulary-parallel token log-probs and entropy (reference:
``lumenrl/utils/vocab_parallel.py:32-88``, which calls Megatron's
``vocab_parallel_cross_entropy``).

Each rank of a tensor-parallel group holds rows [v0, v0 + Vs) of the LM head
and computes the logits of every token for its slice only.  Per token, the
global log-sum-exp, the target logit and (for the entropy) the softmax mean
of the logits are assembled from per-slice partials with three all-reduces of
[T]-sized vectors (max, then sum of exp and the two moments, then the target
logit), so a [T, V] logit matrix never exists on one rank.  The backward
recomputes the slice's logits in row chunks: dlogits = upstream gradient x
(one-hot of the target within the slice - softmax), plus the entropy term
-p (z - E[z]); the input gradient dh = dlogits W_slice is summed over the
group, the weight gradient of the slice stays local (accumulated into
``main_grad`` when the weight has one).
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist
from torch import Tensor

from lumenrl_b200 import ops


def _chunks(T: int, rows: int):
    for a in range(0, T, rows):
        yield a, min(T, a + rows)


class _VocabParallelLogProb(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, w, w_handle, targets, v0, group, inv_t, want_entropy, rows):
        T = h.shape[0]
        Vs = w.shape[0]
        dev = h.device
        m = torch.full((T,), float("-inf"), dtype=torch.float32, device=dev)
        for a, b in _chunks(T, rows):
            m[a:b] = (ops.mm_nt(h[a:b], w).float() * inv_t).amax(-1)
        dist.all_reduce(m, op=dist.ReduceOp.MAX, group=group)
        s = torch.zeros(T, dtype=torch.float32, device=dev)
        ez = torch.zeros(T, dtype=torch.float32, device=dev)
        zt = torch.zeros(T, dtype=torch.float32, device=dev)
        local = (targets >= v0) & (targets < v0 + Vs)
        idx = (targets - v0).clamp(0, Vs - 1)
        for a, b in _chunks(T, rows):
            z = ops.mm_nt(h[a:b], w).float() * inv_t
            e = torch.exp(z - m[a:b, None])
            s[a:b] = e.sum(-1)
            if want_entropy:
                ez[a:b] = (e * z).sum(-1)
            zt[a:b] = torch.where(local[a:b], z.gather(1, idx[a:b, None]).squeeze(1), torch.zeros_like(zt[a:b]))
        red = torch.stack([s, ez, zt])
        dist.all_reduce(red, group=group)
        s, ez, zt = red[0], red[1], red[2]
        lse = m + torch.log(s)
        logp = zt - lse
        mean_z = ez / s
        ent = lse - mean_z if want_entropy else None
        ctx.save_for_backward(h, w, targets, lse, mean_z)
        ctx.w_handle, ctx.v0, ctx.group, ctx.inv_t, ctx.rows, ctx.want_entropy = w_handle, v0, group, inv_t, rows, \
            want_entropy
        ctx.mark_non_differentiable(lse)
        return logp, (ent if ent is not None else torch.zeros_like(logp))

    @staticmethod
    def backward(ctx, g_logp, g_ent):
        h, w, targets, lse, mean_z = ctx.saved_tensors
        T, Vs = h.shape[0], w.shape[0]
        v0, inv_t = ctx.v0, ctx.inv_t
        local = (targets >= v0) & (targets < v0 + Vs)
        idx = (targets - v0).clamp(0, Vs - 1)
        g_logp = g_logp.float() if g_logp is not None else torch.zeros(T, device=h.device)
        use_ent = ctx.want_entropy and g_ent is not None
        dh = torch.zeros(h.shape, dtype=torch.float32, device=h.device)
        dw = torch.zeros(w.shape, dtype=torch.float32, device=w.device)
        for a, b in _chunks(T, ctx.rows):
            z = ops.mm_nt(h[a:b], w).float() * inv_t
            p = torch.exp(z - lse[a:b, None])
            dz = -p * g_logp[a:b, None]
            hit = local[a:b]
            rows_hit = torch.nonzero(hit, as_tuple=True)[0]
            dz[rows_hit, idx[a:b][rows_hit]] += g_logp[a:b][rows_hit]
            if use_ent:
                dz -= p * (z - mean_z[a:b, None]) * g_ent[a:b, None].float()
            dz *= inv_t
            dh[a:b] = dz @ w.float()
            dw += dz.t() @ h[a:b].float()
        dist.all_reduce(dh, group=ctx.group)
        wh = ctx.w_handle
        dw_out = None
        if getattr(wh, "main_grad", None) is not None:
            wh.main_grad += dw.to(wh.main_grad.dtype)
        else:
            dw_out = dw.to(w.dtype)
        return dh.to(h.dtype), None, dw_out, None, None, None, None, None, None


def vocab_parallel_token_logprob(hidden: Tensor, w_slice: Tensor, targets: Tensor, vocab_start: int, group=None,
                                 temperature: float = 1.0, want_entropy: bool = False,
                                 rows: int = 4096) -> tuple[Tensor, Optional[Tensor]]:
    """log p(target) and (optionally) the entropy per row of ``hidden`` [T, H]
    under the LM head whose rows [vocab_start, vocab_start + Vs) are
    ``w_slice`` [Vs, H] on this rank of ``group``.  Every rank of the group
    passes the same ``hidden`` and ``targets`` and gets the same results."""
    inv_t = 1.0 / max(float(temperature), 1e-6)
    logp, ent = _VocabParallelLogProb.apply(hidden, w_slice.detach(), w_slice, targets.long(), int(vocab_start),
                                            group, inv_t, bool(want_entropy), int(rows))
    return logp, (ent if want_entropy else None)


def vocab_slice(vocab_size: int, rank: int, size: int) -> tuple[int, int]:
    """[start, end) of this rank's LM-head rows (the last slice takes the remainder)."""
    per = -(-vocab_size // size)
    return min(rank * per, vocab_size), min((rank + 1) * per, vocab_size)
