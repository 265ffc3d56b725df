"""Custom ops: one function per hot op, autograd-aware.

On CUDA tensors every op here runs a hand-written sm_100a kernel from the
in-tree extension ``lumenrl_b200._C`` (sources under ``csrc/``); if the
extension is missing on a GPU machine the call raises instead of silently
falling back.  CPU tensors use the fp32 PyTorch definitions in
``ops.reference`` (these are also the oracles of the kernel tests).
"""

from __future__ import annotations

import math
from typing import Optional

import os

import torch
from torch import Tensor

from lumenrl_b200.ops import reference as ref
from lumenrl_b200.ops.ext import ext, has_ext  # noqa: F401

__all__ = [
    "rmsnorm", "add_rmsnorm", "qk_norm_rope", "swiglu", "linear", "attention_varlen", "paged_decode_attention",
    "token_logprob", "group_advantage", "ppo_clip_loss", "sample_tokens", "sample_tokens_device", "kv_cache_append", "embedding",
]


def _cuda(*ts) -> bool:
    return any(t is not None and t.is_cuda for t in ts)


# ---------------------------------------------------------------------------
# gradient sinks: weights keep an fp32 ``main_grad`` view into the flat fp32
# gradient buffer; kernels and GEMMs accumulate straight into it.
# ---------------------------------------------------------------------------

def _accum_main_grad(w: Tensor, g: Tensor) -> None:
    mg = getattr(w, "main_grad", None)
    if mg is None:
        if w.grad is None:
            w.grad = g.to(w.dtype)
        else:
            w.grad += g.to(w.dtype)
    else:
        mg += g.to(mg.dtype)


# ---------------------------------------------------------------------------
# Linear: y = x @ W^T, wgrad accumulated in fp32 into W.main_grad
# ---------------------------------------------------------------------------

# Training GEMMs: "own" runs the CTA-pair tcgen05 kernel (csrc/gemm/gemm_2sm.cu)
# for the forward, dgrad and wgrad of every linear; "cublas" is the library
# path kept for A/B measurements (LRL_TRAIN_GEMM=cublas).
TRAIN_GEMM = os.environ.get("LRL_TRAIN_GEMM", "own")


def _pair_ok(*ts) -> bool:
    return (TRAIN_GEMM == "own" and all(t.is_cuda and t.dtype == torch.bfloat16 and t.dim() == 2 and
                                        t.stride(1) == 1 and t.shape[1] % 8 == 0 and t.stride(0) % 8 == 0
                                        for t in ts))


def mm_nt(x: Tensor, w: Tensor) -> Tensor:
    """x [T, K] @ w[N, K]^T -> bf16 [T, N] (forward of a linear)."""
    if _pair_ok(x, w):
        return ext().gemm2sm(x, False, w, False, None, 0, 0)
    return x @ w.t()


def mm_nn(dy: Tensor, w: Tensor) -> Tensor:
    """dy [T, N] @ w [N, K] -> bf16 [T, K] (dgrad: the weight is read MN-major)."""
    if _pair_ok(dy, w):
        return ext().gemm2sm(dy, False, w, True, None, 0, 0)
    return dy @ w


def mm_tn_acc(acc: Tensor, dy: Tensor, x: Tensor) -> None:
    """acc [N, K] (fp32) += dy[T, N]^T @ x[T, K] (wgrad into main_grad)."""
    if _pair_ok(dy, x) and acc.is_contiguous():
        ext().gemm2sm(dy, True, x, True, acc, 2, 0)
    elif acc.is_cuda:
        torch.addmm(acc, dy.t(), x, out_dtype=torch.float32, out=acc)
    else:
        acc += dy.t().float() @ x.float()


class _Linear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x: Tensor, w: Tensor, w_handle: Tensor):
        ctx.save_for_backward(x, w)
        ctx.w_handle = w_handle
        if x.is_cuda:
            x2 = x.reshape(-1, x.shape[-1])
            return mm_nt(x2, w).view(*x.shape[:-1], w.shape[0])
        return x @ w.t()

    @staticmethod
    def backward(ctx, dy: Tensor):
        x, w = ctx.saved_tensors
        wh = ctx.w_handle
        mg = getattr(wh, "main_grad", None)
        dy2, x2 = dy.reshape(-1, dy.shape[-1]), x.reshape(-1, x.shape[-1])
        if dy.is_cuda:
            dy2 = dy2.contiguous()
            dx = mm_nn(dy2, w).view(*dy.shape[:-1], w.shape[1])
            if mg is not None:
                # bf16 x bf16 -> fp32 accumulate (beta = 1) into the flat
                # gradient buffer: no bf16 weight-grad tensor is ever allocated.
                mm_tn_acc(mg, dy2, x2)
            else:
                acc = torch.zeros(w.shape, dtype=torch.float32, device=w.device)
                mm_tn_acc(acc, dy2, x2.contiguous())
                _accum_main_grad(wh, acc)
            return dx, None, None
        dx = dy @ w
        _accum_main_grad(wh, dy2.t().float() @ x2.float())
        return dx, None, None


def linear(x: Tensor, w: Tensor) -> Tensor:
    if not torch.is_grad_enabled() or not w.requires_grad:
        if x.is_cuda:
            return mm_nt(x.reshape(-1, x.shape[-1]), w).view(*x.shape[:-1], w.shape[0])
        return x @ w.t()
    return _Linear.apply(x, w.detach(), w)


class _LinearFP32(torch.autograd.Function):
    """fp32 y = x @ W^T (router gates); wgrad accumulated into main_grad."""

    @staticmethod
    def forward(ctx, x, w, w_handle):
        xf, wf = x.float(), w.float()
        ctx.save_for_backward(xf, wf)
        ctx.w_handle, ctx.x_dtype = w_handle, x.dtype
        return xf @ wf.t()

    @staticmethod
    def backward(ctx, dy):
        xf, wf = ctx.saved_tensors
        dy = dy.float()
        _accum_main_grad(ctx.w_handle, dy.reshape(-1, dy.shape[-1]).t() @ xf.reshape(-1, xf.shape[-1]))
        return (dy @ wf).to(ctx.x_dtype), None, None


def linear_fp32(x: Tensor, w: Tensor) -> Tensor:
    if not torch.is_grad_enabled() or not w.requires_grad:
        return x.float() @ w.float().t()
    return _LinearFP32.apply(x, w.detach(), w)


# ---------------------------------------------------------------------------
# RMSNorm (optionally fused with the residual add that precedes it)
# ---------------------------------------------------------------------------

class _RMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x: Tensor, w: Tensor, w_handle: Tensor, eps: float):
        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        y, rstd = ext().rmsnorm_fwd(x2, w, eps)
        ctx.save_for_backward(x2, w, rstd)
        ctx.w_handle, ctx.shape = w_handle, shape
        return y.view(shape)

    @staticmethod
    def backward(ctx, dy: Tensor):
        x2, w, rstd = ctx.saved_tensors
        dw = torch.zeros(w.shape, dtype=torch.float32, device=w.device)
        dx = ext().rmsnorm_bwd(dy.reshape(x2.shape).contiguous(), x2, w, rstd, dw)
        _accum_main_grad(ctx.w_handle, dw)
        return dx.view(ctx.shape), None, None, None


def rmsnorm(x: Tensor, w: Tensor, eps: float) -> Tensor:
    if not _cuda(x):
        return ref.rmsnorm(x, w, eps)
    if torch.is_grad_enabled() and (x.requires_grad or w.requires_grad):
        return _RMSNorm.apply(x, w.detach(), w, eps)
    shape = x.shape
    y, _ = ext().rmsnorm_fwd(x.reshape(-1, shape[-1]).contiguous(), w, eps)
    return y.view(shape)


class _AddRMSNorm(torch.autograd.Function):
    """(rmsnorm(x + r), x + r) in one kernel; the backward adds the gradient of
    the sum output inside the RMSNorm backward kernel, so neither direction
    launches a separate add."""

    @staticmethod
    def forward(ctx, x: Tensor, r: Tensor, w: Tensor, w_handle: Tensor, eps: float):
        shape = x.shape
        y, s, rstd = ext().add_rmsnorm_fwd(x.reshape(-1, shape[-1]), r.reshape(-1, shape[-1]), w, eps)
        ctx.save_for_backward(s, w, rstd)
        ctx.w_handle, ctx.shape = w_handle, shape
        return y.view(shape), s.view(shape)

    @staticmethod
    def backward(ctx, dy: Tensor, ds: Tensor):
        s, w, rstd = ctx.saved_tensors
        dw = torch.zeros(w.shape, dtype=torch.float32, device=w.device)
        dres = None if ds is None else ds.reshape(s.shape).contiguous()
        if dy is None:
            dy = torch.zeros_like(s)
        dx = ext().rmsnorm_bwd(dy.reshape(s.shape).contiguous(), s, w, rstd, dw, dres)
        _accum_main_grad(ctx.w_handle, dw)
        dx = dx.view(ctx.shape)
        return dx, dx, None, None, None


def add_rmsnorm(x: Tensor, residual: Optional[Tensor], w: Tensor, eps: float) -> tuple[Tensor, Tensor]:
    """Returns (rmsnorm(x + residual), x + residual); ``residual`` may be None."""
    if residual is None:
        return rmsnorm(x, w, eps), x
    if _cuda(x):
        if torch.is_grad_enabled() and (x.requires_grad or residual.requires_grad or w.requires_grad):
            return _AddRMSNorm.apply(x, residual, w.detach(), w, eps)
        shape = x.shape
        y, s, _ = ext().add_rmsnorm_fwd(x.reshape(-1, shape[-1]), residual.reshape(-1, shape[-1]), w, eps)
        return y.view(shape), s.view(shape)
    s = x + residual
    return rmsnorm(s, w, eps), s


# ---------------------------------------------------------------------------
# QK-RMSNorm + RoPE on a fused QKV projection output
# ---------------------------------------------------------------------------

class _QKNormRope(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv, qw, kw, qw_h, kw_h, positions, inv_freq, nh, nkv, hd, eps):
        q, k, v, rq, rk = ext().qk_norm_rope_fwd(qkv, qw, kw, positions, inv_freq, nh, nkv, hd, eps)
        ctx.save_for_backward(qkv, qw, kw, positions, inv_freq, rq, rk)
        ctx.meta = (qw_h, kw_h, nh, nkv, hd, eps)
        return q, k, v

    @staticmethod
    def backward(ctx, dq, dk, dv):
        qkv, qw, kw, positions, inv_freq, rq, rk = ctx.saved_tensors
        qw_h, kw_h, nh, nkv, hd, eps = ctx.meta
        has_norm = qw.numel() > 0
        dqw = torch.zeros(max(qw.numel(), 1), dtype=torch.float32, device=qkv.device)
        dkw = torch.zeros(max(kw.numel(), 1), dtype=torch.float32, device=qkv.device)
        dqkv = ext().qk_norm_rope_bwd(dq.contiguous(), dk.contiguous(), dv.contiguous(), qkv, qw, kw, positions,
                                      inv_freq, rq, rk, dqw, dkw, nh, nkv, hd, eps)
        if has_norm:
            _accum_main_grad(qw_h, dqw)
            _accum_main_grad(kw_h, dkw)
        return dqkv, None, None, None, None, None, None, None, None, None, None


def qk_norm_rope(qkv: Tensor, qw: Optional[Tensor], kw: Optional[Tensor], positions: Tensor, inv_freq: Tensor,
                 nh: int, nkv: int, hd: int, eps: float) -> tuple[Tensor, Tensor, Tensor]:
    """qkv [T, (nh+2nkv)*hd] -> q [T,nh,hd], k [T,nkv,hd], v [T,nkv,hd]."""
    if not _cuda(qkv):
        ang = positions.float().unsqueeze(-1) * inv_freq.float().to(positions.device).unsqueeze(0)
        return ref.qk_norm_rope(qkv, qw, kw, ang.cos(), ang.sin(), nh, nkv, hd, eps)
    empty = qkv.new_empty(0)
    qw_d = qw.detach() if qw is not None else empty
    kw_d = kw.detach() if kw is not None else empty
    if torch.is_grad_enabled() and qkv.requires_grad:
        return _QKNormRope.apply(qkv, qw_d, kw_d, qw, kw, positions, inv_freq, nh, nkv, hd, eps)
    q, k, v, _, _ = ext().qk_norm_rope_fwd(qkv, qw_d, kw_d, positions, inv_freq, nh, nkv, hd, eps)
    return q, k, v


def qk_norm_rope_cache(qkv: Tensor, qw: Optional[Tensor], kw: Optional[Tensor], positions: Tensor,
                       inv_freq: Tensor, nh: int, nkv: int, hd: int, eps: float, k_cache: Tensor, v_cache: Tensor,
                       slots: Tensor, k_scale: float = 1.0, v_scale: float = 1.0) -> tuple[Tensor, Tensor, Tensor]:
    """Inference path: QK-norm + RoPE that also writes k/v into the paged
    caches at ``slots`` in the same kernel (no separate append)."""
    if not _cuda(qkv):
        q, k, v = qk_norm_rope(qkv, qw, kw, positions, inv_freq, nh, nkv, hd, eps)
        kv_cache_append(k, v, k_cache, v_cache, slots, k_scale, v_scale)
        return q, k, v
    empty = qkv.new_empty(0)
    q, k, v, _, _ = ext().qk_norm_rope_fwd(qkv, qw if qw is not None else empty, kw if kw is not None else empty,
                                           positions, inv_freq, nh, nkv, hd, eps, k_cache, v_cache, slots,
                                           1.0 / k_scale, 1.0 / v_scale)
    return q, k, v


# ---------------------------------------------------------------------------
# SwiGLU
# ---------------------------------------------------------------------------

class _SwiGLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, gu):
        ctx.save_for_backward(gu)
        return ext().swiglu_fwd(gu)

    @staticmethod
    def backward(ctx, dh):
        (gu,) = ctx.saved_tensors
        return ext().swiglu_bwd(dh.contiguous(), gu)


def swiglu(gate_up: Tensor) -> Tensor:
    if not _cuda(gate_up):
        return ref.swiglu(gate_up)
    gu = gate_up.contiguous()
    if torch.is_grad_enabled() and gu.requires_grad:
        return _SwiGLU.apply(gu)
    return ext().swiglu_fwd(gu)


# ---------------------------------------------------------------------------
# Attention
# ---------------------------------------------------------------------------

def attention_varlen(q: Tensor, k: Tensor, v: Tensor, cu_seqlens: Tensor, max_seqlen: int,
                     causal: bool = True, scale: Optional[float] = None) -> Tensor:
    """Packed causal attention, q [T,Hq,D], k/v [T,Hk,D]."""
    if not _cuda(q):
        return ref.attention_varlen(q, k, v, cu_seqlens, causal, scale)
    from lumenrl_b200.ops.attention import flash_attention_varlen
    return flash_attention_varlen(q, k, v, cu_seqlens, max_seqlen, causal, scale)


# decode attention kernel for bf16 caches with 64-token pages: "tma" (pages
# streamed by a producer warp with cp.async.bulk.tensor; 5.85 vs 5.31 TB/s at
# 64 x 1.5K context) or "cpasync" (the original kernel)
DECODE_ATTN = os.environ.get("LRL_DECODE_ATTN", "tma")


def _tma_ok(q: Tensor, k_cache: Tensor) -> bool:
    return (DECODE_ATTN == "tma" and q.is_cuda and k_cache.dtype == torch.bfloat16 and k_cache.dim() == 4
            and k_cache.shape[1] == 64 and k_cache.shape[3] == 128 and k_cache.is_contiguous())


def paged_decode_attention(q: Tensor, k_cache: Tensor, v_cache: Tensor, block_table: Tensor, seq_lens: Tensor,
                           scale: float, k_scale: float = 1.0, v_scale: float = 1.0, max_len: int = 0) -> Tensor:
    """q [B,Hq,D] against the paged caches; ``max_len`` (static upper bound of
    seq_lens, 0 = block-table capacity) sizes the context split without a
    device->host read, so the call is CUDA-graph safe."""
    if not _cuda(q):
        return ref.paged_decode_attention(q, k_cache.to(q.dtype) * k_scale if k_cache.dtype != q.dtype else k_cache,
                                          v_cache.to(q.dtype) * v_scale if v_cache.dtype != q.dtype else v_cache,
                                          block_table, seq_lens, scale)
    if _tma_ok(q, k_cache):
        return ext().paged_decode_attn_tma(q, k_cache, v_cache, block_table, seq_lens, scale * k_scale, v_scale,
                                           max_len)
    return ext().paged_decode_attn(q, k_cache, v_cache, block_table, seq_lens, scale, k_scale, v_scale, max_len)


def shared_prefix_group(n: int, gqa: int, limit: int = 64) -> int:
    """Largest divisor of the GRPO group size ``n`` whose rows x GQA heads fit
    one shared-prefix attention CTA (<= ``limit`` MMA rows); 1 = no sharing."""
    for g in range(n, 0, -1):
        if n % g == 0 and g * gqa <= limit:
            return g
    return 1


def paged_decode_attention_shared(q: Tensor, k_cache: Tensor, v_cache: Tensor, block_table: Tensor,
                                  seq_lens: Tensor, prefix_len: Tensor, group: int, scale: float,
                                  k_scale: float = 1.0, v_scale: float = 1.0, max_prefix: int = 0,
                                  max_suffix: int = 0) -> Tensor:
    """Decode attention where rows ``[g*group, (g+1)*group)`` share their first
    ``prefix_len[row]`` tokens (the same whole KV blocks, e.g. a GRPO prompt).
    The shared part is read from HBM once per group instead of once per row;
    the result equals ``paged_decode_attention``.  ``max_prefix`` /
    ``max_suffix`` are static upper bounds of ``prefix_len`` and
    ``seq_lens - prefix_len`` (0 = block-table capacity), so the call reads no
    device value on the host and is CUDA-graph safe."""
    if not _cuda(q):
        return paged_decode_attention(q, k_cache, v_cache, block_table, seq_lens, scale, k_scale, v_scale)
    if _tma_ok(q, k_cache):
        return ext().paged_decode_attn_shared_tma(q, k_cache, v_cache, block_table, seq_lens, prefix_len, group,
                                                  scale * k_scale, v_scale, max_prefix, max_suffix)
    return ext().paged_decode_attn_shared(q, k_cache, v_cache, block_table, seq_lens, prefix_len, group, scale,
                                          k_scale, v_scale, max_prefix, max_suffix)


def kv_cache_append(k: Tensor, v: Tensor, k_cache: Tensor, v_cache: Tensor, slots: Tensor,
                    k_scale: float = 1.0, v_scale: float = 1.0) -> None:
    """Write k/v rows [T,Hk,D] into the paged caches at flat slot indices."""
    if not _cuda(k):
        bs = k_cache.shape[1]
        flat_k = k_cache.view(-1, *k_cache.shape[2:])
        flat_v = v_cache.view(-1, *v_cache.shape[2:])
        flat_k[slots.long()] = (k.float() / k_scale).to(k_cache.dtype)
        flat_v[slots.long()] = (v.float() / v_scale).to(v_cache.dtype)
        return
    ext().kv_append(k, v, k_cache, v_cache, slots, 1.0 / k_scale, 1.0 / v_scale)


# ---------------------------------------------------------------------------
# Token log-prob (+ entropy) from hidden states and the LM head, chunked so
# full logits never exist; backward recomputes each chunk.
# ---------------------------------------------------------------------------

FUSED_LOGPROB_ROWS = 16384   # rows per fused call (its per-tile partials: rows x vocab/256 x 16 B)


def _logprob_forward(hidden: Tensor, w: Tensor, targets: Tensor, inv_temp: float, chunk: int):
    """(logp, entropy, lse) per row.  On the pair GEMM the log-softmax
    reduction runs in the GEMM epilogue and logits are never written;
    otherwise bf16 logits are materialised per ``chunk`` rows."""
    T = hidden.shape[0]
    if _pair_ok(hidden, w) and targets.dtype == torch.long:
        outs = [ext().gemm2sm_logprob(hidden[a: a + FUSED_LOGPROB_ROWS], w,
                                      targets[a: a + FUSED_LOGPROB_ROWS].contiguous(), inv_temp)
                for a in range(0, T, FUSED_LOGPROB_ROWS)]
        if len(outs) == 1:
            return tuple(outs[0])
        return tuple(torch.cat([o[i] for o in outs]) for i in range(3))
    logp = torch.empty(T, dtype=torch.float32, device=hidden.device)
    ent = torch.empty(T, dtype=torch.float32, device=hidden.device)
    lse = torch.empty(T, dtype=torch.float32, device=hidden.device)
    for a in range(0, T, chunk):
        b = min(T, a + chunk)
        ext().logprob_fwd(mm_nt(hidden[a:b], w), targets[a:b].contiguous(), inv_temp, logp[a:b], ent[a:b],
                          lse[a:b])
    return logp, ent, lse


class _TokenLogProb(torch.autograd.Function):
    @staticmethod
    def forward(ctx, hidden, w, w_handle, targets, inv_temp, chunk, want_entropy):
        logp, ent, lse = _logprob_forward(hidden, w, targets, inv_temp, chunk)
        ctx.save_for_backward(hidden, w, targets, lse, ent)
        ctx.meta = (w_handle, inv_temp, chunk, want_entropy)
        return logp, ent

    @staticmethod
    def backward(ctx, dlogp, dent):
        hidden, w, targets, lse, ent = ctx.saved_tensors
        w_handle, inv_temp, chunk, want_entropy = ctx.meta
        T = hidden.shape[0]
        dh = torch.empty_like(hidden)
        dlogp = dlogp.float().contiguous() if dlogp is not None else torch.zeros(T, device=hidden.device)
        dent = dent.float().contiguous() if (dent is not None and want_entropy) else None
        mg = getattr(w_handle, "main_grad", None)
        for a in range(0, T, chunk):
            b = min(T, a + chunk)
            logits = mm_nt(hidden[a:b], w)
            # in place: logits -> dL/dlogits (bf16)
            ext().logprob_bwd(logits, targets[a:b], lse[a:b], dlogp[a:b],
                              dent[a:b] if dent is not None else None, inv_temp,
                              ent[a:b] if dent is not None else None)
            dh[a:b] = mm_nn(logits, w)
            if mg is not None:
                mm_tn_acc(mg, logits, hidden[a:b])
            else:
                _accum_main_grad(w_handle, logits.t().float() @ hidden[a:b].float())
        return dh, None, None, None, None, None, None


def token_logprob(hidden: Tensor, lm_head: Tensor, targets: Tensor, temperature: float = 1.0,
                  chunk: int = 2048, want_entropy: bool = True) -> tuple[Tensor, Optional[Tensor]]:
    """log softmax(hidden @ W^T / T)[target] and the entropy, per row."""
    if not _cuda(hidden):
        logits = hidden @ lm_head.t()
        return ref.token_logprob_from_logits(logits, targets, temperature, want_entropy)
    inv_t = 1.0 / float(temperature)
    if torch.is_grad_enabled() and (hidden.requires_grad or lm_head.requires_grad):
        logp, ent = _TokenLogProb.apply(hidden, lm_head.detach(), lm_head, targets.contiguous(), inv_t, chunk,
                                        want_entropy)
        return logp, (ent if want_entropy else None)
    logp, ent, _ = _logprob_forward(hidden, lm_head, targets, inv_t, chunk)
    return logp, (ent if want_entropy else None)


# ---------------------------------------------------------------------------
# RL math kernels
# ---------------------------------------------------------------------------

def group_advantage(rewards: Tensor, group: int, unbiased: bool = False, eps: float = 1e-8) -> Tensor:
    if not _cuda(rewards):
        return ref.group_advantage(rewards, group, unbiased, eps)
    if rewards.shape[0] % group:
        raise ValueError(f"Batch size {rewards.shape[0]} not divisible by num_generations={group}.")
    return ext().group_adv(rewards.float().contiguous(), group, unbiased, eps)


class _PPOClip(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logp, old, adv, mask, is_w, clip_low, clip_high, clip_c, denom):
        loss, dlogp = ext().ppo_clip_fwd_bwd(logp.contiguous(), old.float().contiguous(), adv.float().contiguous(),
                                             mask.float().contiguous(), is_w, clip_low, clip_high, clip_c, denom)
        ctx.save_for_backward(dlogp)
        return loss

    @staticmethod
    def backward(ctx, g):
        (dlogp,) = ctx.saved_tensors
        return dlogp * g, None, None, None, None, None, None, None, None


def ppo_clip_loss(logp: Tensor, old: Tensor, adv: Tensor, mask: Tensor, clip_low: float, clip_high: float,
                  clip_c: float = 0.0, is_w: Optional[Tensor] = None, denom: Optional[float] = None) -> Tensor:
    """DAPO token-level clipped surrogate: sum(masked per-token loss) / denom
    (denom defaults to the mask count).  Forward computes d(loss)/d(logp) in
    the same pass; backward is a scale."""
    if not _cuda(logp):
        return ref.ppo_clip_token_loss(logp, old, adv, mask, clip_low, clip_high, clip_c, is_w, denom)
    if denom is None:
        denom = -1.0
    isw = is_w.float().contiguous() if is_w is not None else None
    return _PPOClip.apply(logp, old, adv, mask, isw, float(clip_low), float(clip_high), float(clip_c), float(denom))


def sample_tokens_device(logits: Tensor, temperature: float, top_p: float, row_seed: Tensor,
                         step: Tensor) -> tuple[Tensor, Tensor]:
    """Sample one token per row from softmax(logits / T) restricted to the
    top-p nucleus; returns (token ids int64, log-prob of the sampled token
    under softmax(logits / T)).

    Randomness is a counter-based stream keyed by (row_seed[row], step,
    vocab index), so a row's draw does not depend on batch composition and
    the call can live inside a CUDA graph (seed/step are device tensors).
    ``step`` holds one counter for all rows or one per row."""
    inv_t = 1.0 / max(float(temperature), 1e-6)
    if not _cuda(logits):
        z = logits.float() * inv_t
        lp = torch.log_softmax(z, -1)
        toks = []
        per_row = step.numel() > 1
        for r in range(z.shape[0]):
            g = torch.Generator(device="cpu").manual_seed(int(row_seed[r]) * 1000003 + int(step[r if per_row else 0]))
            row = lp[r]
            if top_p < 1.0:
                srt, idx = torch.sort(row, descending=True)
                p = srt.exp()
                keep = (p.cumsum(-1) - p) < top_p
                probs = torch.where(keep, p, torch.zeros_like(p))
                pick = torch.multinomial(probs / probs.sum(), 1, generator=g)
                toks.append(idx[pick])
            else:
                toks.append(torch.multinomial(row.exp(), 1, generator=g))
        tok = torch.cat(toks).long()
        return tok, lp.gather(-1, tok.unsqueeze(-1)).squeeze(-1)
    tok, lp = ext().sample(logits.contiguous(), inv_t, float(top_p), row_seed, step)
    return tok, lp


def sample_tokens(logits: Tensor, temperature: float, top_p: float, seed: int, offset: int) -> tuple[Tensor, Tensor]:
    rows = torch.arange(logits.shape[0], device=logits.device, dtype=torch.long) + int(seed) * 65536
    step = torch.full((1,), int(offset), device=logits.device, dtype=torch.long)
    return sample_tokens_device(logits, temperature, top_p, rows, step)


def embedding(ids: Tensor, table: Tensor) -> Tensor:
    return torch.nn.functional.embedding(ids, table)


def inv_freq_table(head_dim: int, theta: float, scaling: dict | None, device) -> Tensor:
    return ref.rope_inv_freq(head_dim, theta, scaling).to(device)


def softmax_scale(head_dim: int) -> float:
    return 1.0 / math.sqrt(head_dim)


# ---------------------------------------------------------------------------
# tcgen05 GEMM (hand-written sm_100a kernel)
# ---------------------------------------------------------------------------

def tc_gemm(a: Tensor, b: Tensor, out: Optional[Tensor] = None, accumulate: bool = False,
            out_dtype: torch.dtype = torch.bfloat16, bn: int = 0) -> Tensor:
    """C = a @ b.T with a [M,K], b [N,K] bf16 on the tensor cores (TMA + tcgen05
    + TMEM).  ``accumulate``: out (fp32 [M,N]) += a @ b.T."""
    if not _cuda(a):
        r = a.float() @ b.float().t()
        if accumulate:
            out += r
            return out
        return r.to(out_dtype)
    if accumulate:
        return ext().tc_gemm(a, b, out, 2, bn)
    return ext().tc_gemm(a, b, None, 0 if out_dtype == torch.bfloat16 else 1, bn)


def skinny_linear(x: Tensor, w: Tensor, ksplit: int = 0) -> Tensor:
    """x [M, K] @ w[N, K]^T for decode-size M (<= 256) on the weight-streaming
    tcgen05 kernel (operands swapped, K split over a cluster, no library GEMM)."""
    return ext().skinny_gemm(x, w, ksplit)


# decode-step linears: "cublas" (default), "skinny" (own weight-streaming
# kernel) or "auto" (skinny for weights up to 64 M elements, where it is ahead
# of cuBLAS in isolation at M=64: 12.4 vs 18.2 us on 4096x4096, 15.3 vs 17.9
# on 6144x4096; inside the CUDA-graph decode step "auto" measured 1.4 % slower
# than all-cuBLAS, 5.72 vs 5.64 ms per step, hence the default)
DECODE_GEMM = os.environ.get("LRL_DECODE_GEMM", "auto")


def decode_linear(x: Tensor, w: Tensor) -> Tensor:
    """No-grad linear of the rollout decode step (M = live sequences).
    ``LRL_DECODE_GEMM``: ``sk`` the persistent stream-K weight-streaming
    kernel (csrc/gemm/skinny_sk.cu), ``skinny`` the one-tile-per-CTA kernel
    (skinny_gemm.cu), ``cublas``, or ``auto``: the stream-K kernel for the
    LM head (N >= 64 K rows: 208.7 us vs cuBLAS 211.6 at M = 64), the
    one-tile kernel up to 64 M weight elements (qkv, o, w2), cuBLAS between
    (w13: its split tiles make the stream-K tail cost more than it saves)."""
    mode = DECODE_GEMM
    if mode == "auto":
        mode = "sk" if w.shape[0] >= 65536 else ("skinny" if w.numel() <= (64 << 20) else "cublas")
    ok = (x.is_cuda and x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16 and x.dim() == 2
          and x.shape[1] % 8 == 0 and x.is_contiguous() and w.is_contiguous())
    if mode == "sk" and ok and x.shape[0] <= 128:
        return ext().skinny_sk(x, w, 0)
    if mode in ("skinny", "sk") and ok and x.shape[0] <= 256:
        return ext().skinny_gemm(x, w, 0)
    return x @ w.t()


def tc_gemm_status() -> int:
    """Error word of the tcgen05 GEMMs since the last call (0 = no error); a
    non-zero value names the role whose bounded wait expired."""
    return int(ext().tc_gemm_status())


_FP8_ERR: dict = {}


def fp8_gemm_blockwise(x: Tensor, qw: Tensor, sw: Tensor, qx: Optional[Tensor] = None,
                       sx: Optional[Tensor] = None) -> Tensor:
    """W8A8 block-scaled GEMM: bf16 x [M,K] (quantised here to E4M3 with 1x128
    scales unless given) times E4M3 weights qw [N,K] with 128x128 scales sw,
    on the tcgen05 kind::f8f6f4 kernel; returns bf16 [M, N]."""
    if qx is None:
        from lumenrl_b200.quant.fp8 import quant_act_1x128
        qx, sx = quant_act_1x128(x.reshape(-1, x.shape[-1]).contiguous())
    if not _cuda(qx):
        from lumenrl_b200.quant.fp8 import dequant_128x128, dequant_1x128
        return (dequant_1x128(qx, sx) @ dequant_128x128(qw, sw).t()).to(torch.bfloat16)
    dev = qx.device
    if dev not in _FP8_ERR:
        _FP8_ERR[dev] = torch.zeros(1, dtype=torch.int32, device=dev)
    out = ext().fp8_gemm(qx, sx.contiguous(), qw, sw.contiguous(), _FP8_ERR[dev])
    return out.view(*x.shape[:-1], qw.shape[0]) if x is not None else out


FP8_DECODE_GEMM = os.environ.get("LRL_FP8_DECODE_GEMM", "stream")


def fp8_decode_linear(x: Tensor, qw: Tensor, sw: Tensor) -> Tensor:
    """W8A8 linear of the FP8 rollout's decode step (M = live sequences <= 64):
    one activation-quantiser launch (1x128 E4M3 blocks, the rule of
    ``quant_act_1x128``) and the persistent stream-K weight-streaming kernel
    (csrc/gemm/skinny_fp8.cu), which reads the E4M3 weights once.
    ``LRL_FP8_DECODE_GEMM=gemm`` (or shapes it does not take) use the
    compute-shaped block-scaled GEMM after the separate quantiser."""
    ok = (FP8_DECODE_GEMM == "stream" and x.is_cuda and x.dtype == torch.bfloat16 and x.dim() == 2
          and 1 <= x.shape[0] <= 64 and x.shape[1] % 128 == 0 and x.stride(1) == 1 and x.stride(0) % 4 == 0
          and qw.is_contiguous())
    if ok:
        return ext().skinny_fp8(x, qw, sw.contiguous(), 0)
    return fp8_gemm_blockwise(x, qw, sw)


def fp8_gemm_status() -> int:
    v = 0
    for t in _FP8_ERR.values():
        v = max(v, int(t.item()))
        t.zero_()
    return v
