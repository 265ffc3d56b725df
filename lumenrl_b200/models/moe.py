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


class _GroupedLinearTC(torch.autograd.Function):
    """Grouped expert GEMM on the tcgen05 kernel (``csrc/gemm/grouped_gemm.cu``):
    forward and input gradient are single launches driven by the device-side
    offsets; the weight gradient (a per-expert reduction over that expert's
    tokens) reads the offsets on the host once and accumulates each expert's
    ``dy^T x`` in fp32 into ``main_grad`` with cuBLAS."""

    @staticmethod
    def forward(ctx, x, w, w_handle, offsets_dev):
        from lumenrl_b200.ops.ext import ext
        y = ext().grouped_gemm(x.contiguous(), w.contiguous(), offsets_dev)
        ctx.save_for_backward(x, w, offsets_dev)
        ctx.w_handle = w_handle
        return y

    @staticmethod
    def backward(ctx, dy):
        from lumenrl_b200.ops.ext import ext
        x, w, offs = ctx.saved_tensors
        dy = dy.contiguous()
        dx = ext().grouped_gemm(dy, w.transpose(1, 2).contiguous(), offs)
        off = offs.tolist()
        mg = getattr(ctx.w_handle, "main_grad", None)
        gw = None if mg is not None else torch.zeros(w.shape, dtype=torch.float32, device=w.device)
        for e in range(w.shape[0]):
            a, b = off[e], off[e + 1]
            if b > a:
                tgt = mg[e] if mg is not None else gw[e]
                torch.addmm(tgt, dy[a:b].t(), x[a:b], out_dtype=torch.float32, out=tgt)
        if gw is not None:
            ops._accum_main_grad(ctx.w_handle, gw)
        return dx, None, None, None


def grouped_linear_device(x: Tensor, w: Tensor, offsets_dev: Tensor) -> Tensor:
    """Expert GEMM with device offsets [E+1] int32 (bf16 CUDA tensors,
    N and K of the weights multiples of 128 / 8)."""
    if torch.is_grad_enabled() and w.requires_grad:
        return _GroupedLinearTC.apply(x, w.detach(), w, offsets_dev)
    from lumenrl_b200.ops.ext import ext
    return ext().grouped_gemm(x.contiguous(), w.contiguous(), offsets_dev)


def _use_tc_grouped(h: Tensor, w13: Tensor, w2: Tensor) -> bool:
    return (h.is_cuda and h.dtype == torch.bfloat16 and w13.shape[1] % 128 == 0 and w2.shape[1] % 128 == 0
            and w13.shape[2] % 8 == 0 and w2.shape[2] % 8 == 0 and w13.shape[0] <= 512)


def moe_graph_ok(model) -> bool:
    """True when every MoE layer of ``model`` takes the device path (kernel
    routing and the tcgen05 grouped GEMMs with device offsets), i.e. a decode
    step makes no host read of the routes and can be captured in a graph."""
    a = model.args
    if not a.num_experts:
        return True
    if a.num_experts > 512 or a.num_experts_per_tok > 16:
        return False
    P = model._params
    for i in range(a.num_layers):
        if a.is_moe_layer(i):
            w13, w2 = P[f"layers.{i}.experts_w13"], P[f"layers.{i}.experts_w2"]
            probe = w13.new_empty(0)
            if not _use_tc_grouped(probe, w13, w2):
                return False
    return True


class _NullCtx:
    def save_for_backward(self, *a):
        pass


class _RouteDevice(torch.autograd.Function):
    """Softmax + top-k (+ replay) + expert permutation on the device
    (csrc/ops/moe_route.cu); gradients reach the logits through the routing
    weights and the probabilities (aux loss)."""

    @staticmethod
    def forward(ctx, logits, k, norm, replay):
        from lumenrl_b200.ops.ext import ext
        probs, ids, w, order, token_of, offsets, counts = ext().moe_route(logits.contiguous(), k, norm, replay)
        ctx.save_for_backward(probs, ids, w)
        ctx.norm = norm
        ctx.mark_non_differentiable(ids, order, token_of, offsets, counts)
        return w, probs, ids, order, token_of, offsets, counts

    @staticmethod
    def backward(ctx, dw, dprobs, *_):
        from lumenrl_b200.ops.ext import ext
        probs, ids, w = ctx.saved_tensors
        if dw is None:
            dw = torch.zeros_like(w)
        return ext().moe_route_bwd(probs, ids, w, dw, dprobs, ctx.norm), None, None, None


def route_device(h: Tensor, router_w: Tensor, top_k: int, norm_topk: bool, replay_ids: Optional[Tensor] = None):
    """Device routing: (ids [T,k], weights [T,k], probs [T,E], order, token_of,
    offsets int32 [E+1], counts [E]) -- the permutation the grouped GEMMs use."""
    logits = ops.linear_fp32(h, router_w)
    rep = replay_ids.long().to(h.device).contiguous() if replay_ids is not None else None
    w, probs, ids, order, token_of, offsets, counts = _RouteDevice.apply(logits, int(top_k), bool(norm_topk), rep)
    return ids, w, probs, order, token_of, offsets, counts


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
    w13, w2 = P[pre + "experts_w13"], P[pre + "experts_w2"]
    if _use_tc_grouped(h, w13, w2) and a.num_experts <= 1024 and a.num_experts_per_tok <= 16:
        ids, w, probs, order, token_of, offs, counts = route_device(
            h, P[pre + "router"], a.num_experts_per_tok, a.norm_topk_prob, replay)
    else:
        ids, w, probs = route(h, P[pre + "router"], a.num_experts_per_tok, a.norm_topk_prob, replay)
        offs = None
    rec = getattr(model, "routing_recorder", None)
    if rec is not None:
        rec.record(layer, ids)
    stats = getattr(model, "router_stats", None)
    if stats is not None and torch.is_grad_enabled():   # training steps only
        stats.observe(layer, probs, ids)
    T, k = ids.shape
    if offs is None:
        flat_ids = ids.reshape(-1)
        order = torch.argsort(flat_ids, stable=True)
        counts = torch.bincount(flat_ids, minlength=a.num_experts)
        token_of = order // k
    xs = h[token_of]
    if _use_tc_grouped(h, w13, w2):
        if offs is None:
            offs = torch.zeros(a.num_experts + 1, dtype=torch.int32, device=h.device)
            offs[1:] = torch.cumsum(counts, 0)
        gu = grouped_linear_device(xs, w13, offs)
        ys = grouped_linear_device(ops.swiglu(gu), w2, offs)
    else:
        offsets = [0] + torch.cumsum(counts, 0).tolist()
        gu = grouped_linear(xs, w13, offsets)
        ys = grouped_linear(ops.swiglu(gu), w2, offsets)
    wt = w.reshape(-1)[order].to(ys.dtype).unsqueeze(-1)
    out = torch.zeros_like(h)
    out.index_add_(0, token_of, ys * wt)
    aux = None
    if a.router_aux_loss_coef > 0 and torch.is_grad_enabled():
        aux = a.router_aux_loss_coef * load_balance_loss(probs, ids, a.num_experts)
    return out, aux
