"""Mixture-of-experts block (Qwen3-MoE style) with rollout routing replay.

* Router: fp32 gate GEMM (reference ``lumenrl/moe/router_precision.py:44-150``
  keeps the router in fp32 on both sides to stop expert flips), softmax over
  experts, top-k, renormalised over the k chosen (``norm_topk_prob``).
* R3 replay (reference ``lumenrl/moe/rollout_routing.py:96-112``): when the
  model carries replay ids for this layer, the rollout's expert ids replace
  the top-k selection and the weights are re-gathered from the LIVE softmax,
  so the router still receives gradients.
* Experts: tokens are sorted by expert and run through a grouped SwiGLU MLP
  (``grouped_linear``); outputs are scattered back and weighted.
* Aux load-balancing loss ``E * sum_e f_e * P_e`` scaled by
  ``router_aux_loss_coef``.
"""

from __future__ import annotations

from typing import Optional

import torch
from torch import Tensor

from lumenrl_b200 import ops


class _GroupedLinear(torch.autograd.Function):
    """y[rows of e] = x[rows of e] @ W[e]^T for contiguous expert row groups."""

    @staticmethod
    def forward(ctx, x, w, w_handle, offsets: list[int]):
        y = x.new_empty(x.shape[0], w.shape[1])
        for e in range(w.shape[0]):
            a, b = offsets[e], offsets[e + 1]
            if b > a:
                torch.mm(x[a:b], w[e].t(), out=y[a:b])
        ctx.save_for_backward(x, w)
        ctx.w_handle, ctx.offsets = w_handle, offsets
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w = ctx.saved_tensors
        offsets = ctx.offsets
        dx = torch.zeros_like(x)
        mg = getattr(ctx.w_handle, "main_grad", None)
        gw = None if mg is not None else torch.zeros(w.shape, dtype=torch.float32, device=w.device)
        for e in range(w.shape[0]):
            a, b = offsets[e], offsets[e + 1]
            if b <= a:
                continue
            dx[a:b] = dy[a:b] @ w[e]
            if mg is not None and dy.is_cuda:
                torch.addmm(mg[e], dy[a:b].t(), x[a:b], out_dtype=torch.float32, out=mg[e])
            else:
                (mg if mg is not None else gw)[e] += dy[a:b].t().float() @ x[a:b].float()
        if gw is not None:
            ops._accum_main_grad(ctx.w_handle, gw)
        return dx, None, None, None


def grouped_linear(x: Tensor, w: Tensor, offsets: list[int]) -> Tensor:
    if torch.is_grad_enabled() and w.requires_grad:
        return _GroupedLinear.apply(x, w.detach(), w, offsets)
    return _GroupedLinear.forward(_NullCtx(), x, w, None, offsets)


class _NullCtx:
    def save_for_backward(self, *a):
        pass


def route(h: Tensor, router_w: Tensor, top_k: int, norm_topk: bool,
          replay_ids: Optional[Tensor] = None) -> tuple[Tensor, Tensor, Tensor]:
    """Returns (expert ids [T,k] int64, weights [T,k] fp32, full probs [T,E])."""
    logits = ops.linear_fp32(h, router_w)
    probs = torch.softmax(logits, dim=-1)
    w, ids = torch.topk(probs, top_k, dim=-1)
    if replay_ids is not None:
        from lumenrl_b200.moe.r3 import apply_replay
        ids = apply_replay(probs, ids, replay_ids.long().to(h.device))
        w = probs.gather(-1, ids)
    if norm_topk:
        w = w / w.sum(-1, keepdim=True).clamp_min(1e-20)
    return ids, w, probs


def load_balance_loss(probs: Tensor, ids: Tensor, num_experts: int) -> Tensor:
    T, k = ids.shape
    counts = torch.zeros(num_experts, device=probs.device, dtype=torch.float32)
    counts.index_add_(0, ids.reshape(-1), torch.ones(T * k, device=probs.device))
    f = counts / max(T * k, 1)
    return num_experts * (f * probs.mean(0)).sum()


def moe_forward(model, layer: int, h: Tensor) -> tuple[Tensor, Optional[Tensor]]:
    a = model.args
    P = model._params
    pre = f"layers.{layer}."
    replay = None
    rr = getattr(model, "routing_replay", None)
    if rr is not None:
        replay = rr.lookup(layer, h.shape[0])
    ids, w, probs = route(h, P[pre + "router"], a.num_experts_per_tok, a.norm_topk_prob, replay)
    rec = getattr(model, "routing_recorder", None)
    if rec is not None:
        rec.record(layer, ids)
    T, k = ids.shape
    flat_ids = ids.reshape(-1)
    order = torch.argsort(flat_ids, stable=True)
    counts = torch.bincount(flat_ids, minlength=a.num_experts)
    offsets = [0] + torch.cumsum(counts, 0).tolist()
    token_of = order // k
    xs = h[token_of]
    gu = grouped_linear(xs, P[pre + "experts_w13"], offsets)
    ys = grouped_linear(ops.swiglu(gu), P[pre + "experts_w2"], offsets)
    wt = w.reshape(-1)[order].to(ys.dtype).unsqueeze(-1)
    out = torch.zeros_like(h)
    out.index_add_(0, token_of, ys * wt)
    aux = None
    if a.router_aux_loss_coef > 0 and torch.is_grad_enabled():
        aux = a.router_aux_loss_coef * load_balance_loss(probs, ids, a.num_experts)
    return out, aux
