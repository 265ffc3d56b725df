"""Eagle3 draft-training ops on this package's kernels.

``ttt_attention``: attention of one test-time-training (TTT) step.  Step i's
queries attend causally to the step-0 keys of their sequence and to the i
"diagonal" keys that steps 1..i produced at the same position.  The causal
part is the tcgen05 flash-attention forward (``csrc/attn/fa_fwd.cu``, which
also returns the log-sum-exp); ``csrc/attn/ttt_diag.cu`` merges the diagonal
terms into it by log-sum-exp weights.  The backward is the tcgen05 flash
backward fed the merged output and merged log-sum-exp, plus the diagonal
kernel's share (dQ added in place, dK/dV of each diagonal step).  Reference
behaviour: ``lumenrl/models/eagle3.py:346-407``.

``forward_kl``: per-row KL(teacher || draft) over the draft vocabulary and
top-1 agreement.  Both LM-head GEMMs run on the CTA-pair tcgen05 GEMM, the
row reduction and dKL/dlogits on ``csrc/ops/fkl.cu``; the backward GEMMs read
the stored bf16 dKL/dlogits.  Reference behaviour:
``lumenrl/models/eagle3.py:605-640``.
"""

from __future__ import annotations

import torch
from torch import Tensor

from lumenrl_b200.ops import _accum_main_grad, mm_nn, mm_nt, mm_tn_acc
from lumenrl_b200.ops.ext import ext


def ttt_kernels_ok(q: Tensor) -> bool:
    return q.is_cuda and q.dtype == torch.bfloat16 and q.dim() == 3 and q.shape[-1] == 128


class _TTTAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k0, v0, cu, max_len, scale, *diag):
        q, k0, v0 = q.contiguous(), k0.contiguous(), v0.contiguous()
        nd = len(diag) // 2
        kd = [d.contiguous() for d in diag[:nd]]
        vd = [d.contiguous() for d in diag[nd:]]
        out, lse = ext().fa_fwd(q, k0, v0, cu, max_len, scale)
        if nd:
            out, lse = ext().ttt_diag_fwd(q, out, lse, kd, vd, scale)
        ctx.save_for_backward(q, k0, v0, out, lse, cu, *kd, *vd)
        ctx.meta = (max_len, scale, nd)
        return out

    @staticmethod
    def backward(ctx, dout):
        q, k0, v0, out, lse, cu, *diag = ctx.saved_tensors
        max_len, scale, nd = ctx.meta
        dout = dout.contiguous()
        dq, dk0, dv0 = ext().fa_bwd(dout, q, k0, v0, out, lse, cu, max_len, scale)
        grads = []
        if nd:
            grads = ext().ttt_diag_bwd(dout, q, out, lse, list(diag[:nd]), list(diag[nd:]), dq, scale)
        return (dq, dk0, dv0, None, None, None, *grads)


def ttt_attention(q: Tensor, cache: list, cu_seqlens: Tensor, max_seqlen: int, scale: float) -> Tensor:
    """q [T, H, 128] of TTT step ``len(cache) - 1``; ``cache`` holds the
    (k, v) [T, KVH, 128] of steps 0..i.  bf16 CUDA tensors."""
    k0, v0 = cache[0]
    kd = [k for k, _ in cache[1:]]
    vd = [v for _, v in cache[1:]]
    return _TTTAttention.apply(q, k0, v0, cu_seqlens.to(torch.int32), int(max_seqlen), float(scale), *kd, *vd)


class _ForwardKL(torch.autograd.Function):
    @staticmethod
    def forward(ctx, draft_h, w_draft, w_handle, teacher_h, w_teacher, chunk):
        n = draft_h.shape[0]
        kl = torch.empty(n, dtype=torch.float32, device=draft_h.device)
        hit = torch.empty_like(kl)
        dz = []
        for a in range(0, n, chunk):
            b = min(n, a + chunk)
            zt = mm_nt(teacher_h[a:b], w_teacher)
            zd = mm_nt(draft_h[a:b], w_draft)
            k, h, _ = ext().fkl_fwd(zt, zd)      # zd <- softmax(zd) - softmax(zt)
            kl[a:b] = k
            hit[a:b] = h
            dz.append(zd)
            del zt
        ctx.save_for_backward(draft_h, w_draft)
        ctx.dz, ctx.w_handle, ctx.chunk = dz, w_handle, chunk
        return kl, hit

    @staticmethod
    def backward(ctx, dkl, dhit):
        draft_h, w_draft = ctx.saved_tensors
        n, chunk, wh = draft_h.shape[0], ctx.chunk, ctx.w_handle
        dh = torch.empty_like(draft_h)
        g = dkl.float().contiguous() if dkl is not None else torch.zeros(n, device=draft_h.device)
        mg = getattr(wh, "main_grad", None)
        for i, a in enumerate(range(0, n, chunk)):
            b = min(n, a + chunk)
            dz = ctx.dz[i]
            ext().row_scale_(dz, g[a:b])
            dh[a:b] = mm_nn(dz, w_draft)
            if mg is not None:
                mm_tn_acc(mg, dz, draft_h[a:b])
            elif wh.requires_grad:
                acc = torch.zeros(w_draft.shape, dtype=torch.float32, device=dz.device)
                mm_tn_acc(acc, dz, draft_h[a:b])
                _accum_main_grad(wh, acc)
        ctx.dz = None
        return dh, None, None, None, None, None


def forward_kl(draft_h: Tensor, w_draft: Tensor, teacher_h: Tensor, w_teacher: Tensor,
               chunk: int = 4096) -> tuple[Tensor, Tensor]:
    """Per row: KL(softmax(teacher_h W_t^T) || softmax(draft_h W_d^T)) and
    1.0 where both arg-maxes agree.  bf16 CUDA inputs; gradients reach
    ``draft_h`` and ``w_draft`` (``main_grad`` when the weight has one)."""
    th = teacher_h.to(torch.bfloat16).contiguous()
    wt = w_teacher.to(torch.bfloat16).contiguous()
    dh = draft_h.contiguous()
    if torch.is_grad_enabled() and (draft_h.requires_grad or w_draft.requires_grad):
        return _ForwardKL.apply(dh, w_draft.detach(), w_draft, th, wt, chunk)
    with torch.no_grad():
        return _ForwardKL.forward(_NoCtx(), dh, w_draft, w_draft, th, wt, chunk)


class _NoCtx:
    """Stand-in autograd context for the no-grad forward."""

    def save_for_backward(self, *a):
        pass
