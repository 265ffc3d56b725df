"""Eagle3 speculative-decoding draft model with test-time-training unroll.

Architecture (reference ``lumenrl/models/eagle3.py:46-682``):

* ``fc``: ``3H -> H`` over the concatenated teacher hidden states of three
  auxiliary layers (e.g. 2, 18, 33 of Qwen3-8B); applied once.
* one (or more) decoder layers whose attention input is
  ``[input_norm(token_embeds) ; hidden_norm(h)]`` (2H wide), GQA attention,
  ``o_proj`` back to H with the residual, then a SwiGLU MLP with residual.
* ``length`` TTT steps share one K/V cache: step 0 attends causally over the
  sequence's step-0 keys; step i additionally attends to the i "diagonal"
  keys produced at the SAME position by steps 1..i (the draft's own earlier
  predictions for that position).  RoPE positions advance by one per step.
  Between steps the token ids and the loss mask shift left by one
  (off-policy: ground-truth next tokens), ``h`` carries over.
* loss per step: forward KL from the teacher distribution (teacher LM head on
  the teacher's last hidden state ``step`` positions ahead) to the draft
  distribution, over the draft vocabulary: a fixed subset of the teacher
  vocabulary (``d2t`` maps draft ids to teacher ids).  Steps are weighted by
  ``decay ** step``.

Implementation notes: sequences are packed (``cu_seqlens``); step-0 attention
and the diagonal terms are merged with log-sum-exp weights so the cache never
needs a [T, T] matrix per extra step.
"""

from __future__ import annotations

import math
import os
from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F
from torch import Tensor

from lumenrl_b200 import ops
from lumenrl_b200.ops import reference as ref

# bf16 CUDA tensors take this package's kernels (TTT attention, forward KL,
# GEMMs, norms); LRL_EAGLE_KERNELS=0 keeps the PyTorch path for comparisons
_KERNELS = os.environ.get("LRL_EAGLE_KERNELS", "1") != "0"


class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float = 1e-6) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.eps = eps

    def forward(self, x: Tensor) -> Tensor:
        if _KERNELS and x.is_cuda and x.dtype == torch.bfloat16 and self.weight.dtype == torch.bfloat16:
            return ops.rmsnorm(x, self.weight, self.eps)
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps) * self.weight.float()).to(x.dtype)


def draft_vocab_map(teacher_vocab: int, draft_vocab: int, seed: int = 0) -> Tensor:
    """Fixed seeded subset of the teacher vocabulary, sorted (draft id -> teacher id)."""
    g = torch.Generator().manual_seed(seed)
    return torch.randperm(teacher_vocab, generator=g)[:draft_vocab].sort().values


class Eagle3Layer(nn.Module):
    def __init__(self, hidden: int, heads: int, kv_heads: int, head_dim: int, ffn: int, eps: float,
                 inv_freq: Tensor) -> None:
        super().__init__()
        self.h, self.nh, self.nkv, self.hd = hidden, heads, kv_heads, head_dim
        self.input_norm = RMSNorm(hidden, eps)
        self.hidden_norm = RMSNorm(hidden, eps)
        self.post_norm = RMSNorm(hidden, eps)
        self.wqkv = nn.Linear(2 * hidden, (heads + 2 * kv_heads) * head_dim, bias=False)
        self.wo = nn.Linear(heads * head_dim, hidden, bias=False)
        self.w13 = nn.Linear(hidden, 2 * ffn, bias=False)
        self.w2 = nn.Linear(ffn, hidden, bias=False)
        # fp32 RoPE frequencies, kept out of the module's buffers so that a
        # cast of the module to bf16 does not round them
        self._inv_freq = inv_freq.float()
        self.scale = 1.0 / math.sqrt(head_dim)
        self.eps = eps

    def inv_freq(self, device) -> Tensor:
        if self._inv_freq.device != device:
            self._inv_freq = self._inv_freq.to(device)
        return self._inv_freq

    def _rope(self, x: Tensor, pos: Tensor) -> Tensor:
        ang = pos.float().unsqueeze(-1) * self.inv_freq(x.device).unsqueeze(0)
        return ref.apply_rope(x, ang.cos(), ang.sin())

    def forward(self, emb: Tensor, h: Tensor, pos: Tensor, cu: Tensor, cache: list, max_len: int = 0) -> Tensor:
        T = h.shape[0]
        if _KERNELS and h.is_cuda and h.dtype == torch.bfloat16 and self.hd == 128 and max_len > 0:
            return self._forward_kernels(emb, h, pos, cu, cache, max_len)
        x = torch.cat([self.input_norm(emb), self.hidden_norm(h)], -1)
        qkv = self.wqkv(x)
        q = qkv[:, : self.nh * self.hd].view(T, self.nh, self.hd)
        k = qkv[:, self.nh * self.hd: (self.nh + self.nkv) * self.hd].view(T, self.nkv, self.hd)
        v = qkv[:, (self.nh + self.nkv) * self.hd:].view(T, self.nkv, self.hd)
        step = len(cache)
        q = self._rope(q, pos + step)
        k = self._rope(k, pos + step)
        cache.append((k, v))
        o = cached_tree_attention(q, cache, cu, self.scale)
        h = h + self.wo(o.reshape(T, -1))
        gu = self.w13(self.post_norm(h))
        f = gu.shape[-1] // 2
        return h + self.w2(F.silu(gu[:, :f]) * gu[:, f:])

    def _forward_kernels(self, emb: Tensor, h: Tensor, pos: Tensor, cu: Tensor, cache: list, max_len: int) -> Tensor:
        """Same layer on this package's kernels: RMSNorm, CTA-pair GEMMs,
        RoPE, TTT attention (flash + diagonal merge), SwiGLU."""
        from lumenrl_b200.ops.eagle import ttt_attention
        T = h.shape[0]
        x = torch.cat([ops.rmsnorm(emb, self.input_norm.weight, self.eps),
                       ops.rmsnorm(h, self.hidden_norm.weight, self.eps)], -1)
        qkv = ops.linear(x, self.wqkv.weight)
        step = len(cache)
        q, k, v = ops.qk_norm_rope(qkv, None, None, pos + step, self.inv_freq(h.device), self.nh, self.nkv,
                                   self.hd, self.eps)
        cache.append((k, v))
        o = ttt_attention(q, cache, cu, max_len, self.scale)
        h = h + ops.linear(o.reshape(T, -1), self.wo.weight)
        gu = ops.linear(ops.rmsnorm(h, self.post_norm.weight, self.eps), self.w13.weight)
        return h + ops.linear(ops.swiglu(gu), self.w2.weight)


def cached_tree_attention(q: Tensor, cache: list, cu: Tensor, scale: float, block: int = 1024) -> Tensor:
    """Step-0 causal attention over each packed sequence merged with the
    per-position diagonal keys of steps 1..i, via log-sum-exp weights.
    Query blocks keep the score matrix at [block, T] per head."""
    k0, v0 = cache[0]
    T, H, D = q.shape
    rep = H // k0.shape[1]
    out = torch.empty_like(q)
    cu_l = cu.tolist()
    for s in range(len(cu_l) - 1):
        a, b = cu_l[s], cu_l[s + 1]
        kk = k0[a:b].float().transpose(0, 1).repeat_interleave(rep, 0)   # [H, L, D]
        vv = v0[a:b].float().transpose(0, 1).repeat_interleave(rep, 0)
        for qa in range(a, b, block):
            qb = min(b, qa + block)
            qq = q[qa:qb].float().transpose(0, 1)                         # [H, l, D]
            sc = (qq @ kk.transpose(-1, -2)) * scale                      # [H, l, L]
            qi = torch.arange(qa - a, qb - a, device=q.device)
            ki = torch.arange(0, b - a, device=q.device)
            sc = sc.masked_fill(ki.unsqueeze(0) > qi.unsqueeze(1), float("-inf"))
            diag = []
            for kd, vd in cache[1:]:
                kdd = kd[qa:qb].float().transpose(0, 1).repeat_interleave(rep, 0)   # [H, l, D]
                diag.append(((qq * kdd).sum(-1) * scale, vd[qa:qb].float().transpose(0, 1).repeat_interleave(rep, 0)))
            m = sc.amax(-1)
            for sd, _ in diag:
                m = torch.maximum(m, sd)
            p = torch.exp(sc - m.unsqueeze(-1))
            den = p.sum(-1)
            acc = p @ vv
            for sd, vd in diag:
                w = torch.exp(sd - m)
                den = den + w
                acc = acc + w.unsqueeze(-1) * vd
            out[qa:qb] = (acc / den.unsqueeze(-1)).transpose(0, 1).to(q.dtype)
    return out


class Eagle3Model(nn.Module):
    def __init__(self, hidden: int, teacher_vocab: int, draft_vocab: int, num_heads: int, num_kv_heads: int,
                 head_dim: int = 128, ffn: Optional[int] = None, num_layers: int = 1, length: int = 7,
                 eps: float = 1e-6, rope_theta: float = 1e6, rope_scaling: Optional[dict] = None,
                 vocab_seed: int = 0) -> None:
        super().__init__()
        self.hidden, self.length = hidden, length
        ffn = ffn or 4 * hidden
        inv = ref.rope_inv_freq(head_dim, rope_theta, rope_scaling)
        self.fc = nn.Linear(3 * hidden, hidden, bias=False)
        self.layers = nn.ModuleList([Eagle3Layer(hidden, num_heads, num_kv_heads, head_dim, ffn, eps, inv)
                                     for _ in range(num_layers)])
        self.out_norm = RMSNorm(hidden, eps)
        self.lm_head = nn.Linear(hidden, draft_vocab, bias=False)
        self.register_buffer("d2t", draft_vocab_map(teacher_vocab, draft_vocab, vocab_seed), persistent=True)

    def forward(self, input_ids: Tensor, aux_hidden: Tensor, target_hidden: Tensor, embed_weight: Tensor,
                teacher_lm_head: Tensor, cu_seqlens: Tensor, loss_mask: Tensor, decay: float = 0.8,
                chunk: int = 2048) -> dict:
        """Packed inputs: ``input_ids`` [T], ``aux_hidden`` [T, 3H],
        ``target_hidden`` [T, H] (teacher final-normed), ``loss_mask`` [T]."""
        T = input_ids.shape[0]
        cu = cu_seqlens
        lens = (cu[1:] - cu[:-1])
        lens_h = lens.tolist()
        max_len = max(lens_h) if lens_h else 0
        pos = torch.cat([torch.arange(int(n), device=input_ids.device) for n in lens_h])
        seq_id = torch.repeat_interleave(torch.arange(len(lens), device=input_ids.device), lens)
        kernels = _KERNELS and aux_hidden.is_cuda and aux_hidden.dtype == torch.bfloat16
        h = ops.linear(aux_hidden, self.fc.weight) if kernels else self.fc(aux_hidden)
        ids, mask = input_ids, loss_mask.float()
        w_teacher = teacher_lm_head.index_select(0, self.d2t.to(teacher_lm_head.device))
        caches: list[list] = [[] for _ in self.layers]
        losses, accs = [], []
        total = torch.zeros((), device=h.device)
        for step in range(self.length):
            emb = F.embedding(ids, embed_weight)
            for li, layer in enumerate(self.layers):
                h = layer(emb, h, pos, cu, caches[li], max_len)
            # teacher hidden `step` positions ahead (same sequence only)
            tgt_idx = torch.arange(T, device=h.device) + step
            valid = (tgt_idx < T)
            tgt_idx = tgt_idx.clamp(max=T - 1)
            valid = valid & (seq_id[tgt_idx] == seq_id) & (mask > 0)
            idx = valid.nonzero(as_tuple=True)[0]
            if idx.numel():
                dh = self.out_norm(h).index_select(0, idx)
                th = target_hidden.index_select(0, tgt_idx[idx])
                if kernels:
                    from lumenrl_b200.ops.eagle import forward_kl
                    kl_rows, hit = forward_kl(dh, self.lm_head.weight, th, w_teacher)
                    kl, acc = kl_rows.sum() / idx.numel(), hit.sum() / idx.numel()
                else:
                    kl, acc = self._fkl(dh, th, w_teacher, chunk)
                losses.append(kl)
                accs.append(acc)
                total = total + (decay ** step) * kl
            # shift ids / mask left within each packed sequence
            nxt = torch.arange(T, device=h.device) + 1
            same = (nxt < T)
            nxt = nxt.clamp(max=T - 1)
            same = same & (seq_id[nxt] == seq_id)
            ids = torch.where(same, ids[nxt], torch.zeros_like(ids))
            mask = torch.where(same, mask[nxt], torch.zeros_like(mask))
        return {"loss": total, "losses": losses, "accuracies": accs}

    def _fkl(self, draft_h: Tensor, teacher_h: Tensor, w_teacher: Tensor, chunk: int) -> tuple[Tensor, Tensor]:
        kl_sum = draft_h.new_zeros((), dtype=torch.float32)
        acc = draft_h.new_zeros((), dtype=torch.float32)
        n = draft_h.shape[0]
        for a in range(0, n, chunk):
            b = min(n, a + chunk)
            with torch.no_grad():
                tl = (teacher_h[a:b].to(w_teacher.dtype) @ w_teacher.t()).float()
                tp = tl.softmax(-1)
                tpred = tl.argmax(-1)
            dl = self.lm_head(draft_h[a:b]).float()
            kl_sum = kl_sum + (torch.logsumexp(dl, -1) - (tp * dl).sum(-1) + (tp * tp.clamp_min(1e-30).log()).sum(-1)).sum()
            acc = acc + (dl.argmax(-1) == tpred).float().sum()
        return kl_sum / max(n, 1), acc / max(n, 1)
