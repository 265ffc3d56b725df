"""Plain-PyTorch definitions of every custom op.

These are the numerical oracles the CUDA kernels are tested against, and the
implementation used when tensors live on the CPU (the gloo test tier).  They
favour clarity over speed and compute in fp32.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import Tensor


def rmsnorm(x: Tensor, w: Tensor, eps: float) -> Tensor:
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return (y * w.float()).to(x.dtype)


def rope_cos_sin(positions: Tensor, head_dim: int, theta: float, scaling: dict | None = None) -> tuple[Tensor, Tensor]:
    """cos/sin tables [T, head_dim/2] in fp32 for rotate-half RoPE."""
    inv = rope_inv_freq(head_dim, theta, scaling).to(positions.device)
    ang = positions.float().unsqueeze(-1) * inv.unsqueeze(0)
    return ang.cos(), ang.sin()


def rope_inv_freq(head_dim: int, theta: float, scaling: dict | None = None) -> Tensor:
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim))
    if scaling:
        kind = scaling.get("type")
        if kind == "llama3":
            factor = scaling["factor"]
            lo, hi = scaling.get("low_freq_factor", 1.0), scaling.get("high_freq_factor", 4.0)
            old = scaling.get("original_max_position_embeddings", 8192)
            wavelen = 2 * math.pi / inv
            lo_w, hi_w = old / lo, old / hi
            smooth = (old / wavelen - lo) / (hi - lo)
            scaled = torch.where(wavelen > lo_w, inv / factor, inv)
            mid = (wavelen <= lo_w) & (wavelen >= hi_w)
            inv = torch.where(mid, (1 - smooth) * inv / factor + smooth * inv, scaled)
        elif kind == "yarn":
            factor = scaling["factor"]
            old = scaling.get("original_max_position_embeddings", 4096)
            beta_fast, beta_slow = scaling.get("beta_fast", 32.0), scaling.get("beta_slow", 1.0)

            def dim_of(rot: float) -> float:
                return (head_dim * math.log(old / (rot * 2 * math.pi))) / (2 * math.log(theta))
            low = max(math.floor(dim_of(beta_fast)), 0)
            high = min(math.ceil(dim_of(beta_slow)), head_dim - 1)
            ramp = ((torch.arange(head_dim // 2, dtype=torch.float64) - low) / max(high - low, 1e-3)).clamp(0, 1)
            inv = inv / factor * ramp + inv * (1 - ramp)
    return inv.float()


def apply_rope(x: Tensor, cos: Tensor, sin: Tensor) -> Tensor:
    """x [T, H, D]; rotate-half convention (first half / second half)."""
    d = x.shape[-1] // 2
    xf = x.float()
    x1, x2 = xf[..., :d], xf[..., d:]
    c, s = cos.unsqueeze(1), sin.unsqueeze(1)
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], -1).to(x.dtype)


def qk_norm_rope(qkv: Tensor, qw: Tensor | None, kw: Tensor | None, cos: Tensor, sin: Tensor,
                 nh: int, nkv: int, hd: int, eps: float) -> tuple[Tensor, Tensor, Tensor]:
    T = qkv.shape[0]
    q = qkv[:, : nh * hd].reshape(T, nh, hd)
    k = qkv[:, nh * hd: (nh + nkv) * hd].reshape(T, nkv, hd)
    v = qkv[:, (nh + nkv) * hd:].reshape(T, nkv, hd)
    if qw is not None:
        q = rmsnorm(q, qw, eps)
        k = rmsnorm(k, kw, eps)
    return apply_rope(q, cos, sin), apply_rope(k, cos, sin), v.contiguous()


def swiglu(gate_up: Tensor) -> Tensor:
    f = gate_up.shape[-1] // 2
    g, u = gate_up[..., :f].float(), gate_up[..., f:].float()
    return (F.silu(g) * u).to(gate_up.dtype)


def attention_varlen(q: Tensor, k: Tensor, v: Tensor, cu_seqlens: Tensor, causal: bool = True,
                     scale: float | None = None) -> Tensor:
    """q [T, Hq, D], k/v [T, Hk, D] packed by ``cu_seqlens``; GQA by head repeat."""
    hq, hk, d = q.shape[1], k.shape[1], q.shape[2]
    scale = scale if scale is not None else 1.0 / math.sqrt(d)
    out = torch.empty_like(q)
    cu = cu_seqlens.tolist()
    for i in range(len(cu) - 1):
        a, b = cu[i], cu[i + 1]
        if b <= a:
            continue
        qi = q[a:b].float().transpose(0, 1)
        ki = k[a:b].float().transpose(0, 1).repeat_interleave(hq // hk, 0)
        vi = v[a:b].float().transpose(0, 1).repeat_interleave(hq // hk, 0)
        s = qi @ ki.transpose(-1, -2) * scale
        if causal:
            n = b - a
            s = s.masked_fill(torch.ones(n, n, dtype=torch.bool, device=q.device).triu(1), float("-inf"))
        out[a:b] = (s.softmax(-1) @ vi).transpose(0, 1).to(q.dtype)
    return out


def paged_decode_attention(q: Tensor, k_cache: Tensor, v_cache: Tensor, block_table: Tensor, seq_lens: Tensor,
                           scale: float) -> Tensor:
    """q [B, Hq, D]; caches [num_blocks, block, Hk, D]; block_table [B, max_blocks]."""
    B, hq, d = q.shape
    bs, hk = k_cache.shape[1], k_cache.shape[2]
    out = torch.empty_like(q)
    for i in range(B):
        n = int(seq_lens[i])
        nb = (n + bs - 1) // bs
        blocks = block_table[i, :nb].long()
        kk = k_cache[blocks].reshape(nb * bs, hk, d)[:n].float()
        vv = v_cache[blocks].reshape(nb * bs, hk, d)[:n].float()
        kk = kk.transpose(0, 1).repeat_interleave(hq // hk, 0)
        vv = vv.transpose(0, 1).repeat_interleave(hq // hk, 0)
        s = (q[i].float().unsqueeze(1) @ kk.transpose(-1, -2)).squeeze(1) * scale
        out[i] = (s.softmax(-1).unsqueeze(1) @ vv).squeeze(1).to(q.dtype)
    return out


def token_logprob_from_logits(logits: Tensor, targets: Tensor, temperature: float = 1.0,
                              want_entropy: bool = True) -> tuple[Tensor, Tensor | None]:
    z = logits.float() / temperature
    lse = torch.logsumexp(z, -1)
    logp = z.gather(-1, targets.long().unsqueeze(-1)).squeeze(-1) - lse
    ent = None
    if want_entropy:
        p = torch.softmax(z, -1)
        ent = lse - (p * z).sum(-1)
    return logp, ent


def group_advantage(rewards: Tensor, group: int, unbiased: bool, eps: float) -> Tensor:
    g = rewards.float().view(-1, group)
    return ((g - g.mean(1, keepdim=True)) / g.std(1, unbiased=unbiased, keepdim=True).clamp_min(eps)).reshape(-1)


def ppo_clip_token_loss(logp: Tensor, old: Tensor, adv: Tensor, mask: Tensor, clip_low: float, clip_high: float,
                        clip_c: float, is_w: Tensor | None, denom: float | None) -> Tensor:
    ratio = torch.exp((logp - old).clamp(-20.0, 20.0))
    pg = torch.maximum(-adv * ratio, -adv * ratio.clamp(1.0 - clip_low, 1.0 + clip_high))
    if clip_c > 0:
        pg = torch.where(adv < 0, torch.minimum(-adv * clip_c, pg), pg)
    if is_w is not None:
        pg = pg * is_w
    pg = torch.where(mask.bool(), pg, torch.zeros_like(pg))
    if denom is None:
        denom = float(mask.float().sum().clamp(min=1.0))
    return pg.sum() / denom


def adamw_reference(p32: Tensor, g: Tensor, m: Tensor, v: Tensor, lr: float, beta1: float, beta2: float,
                    eps: float, wd: float, step: int, grad_scale: float) -> None:
    g = g.float() * grad_scale
    m.mul_(beta1).add_(g, alpha=1 - beta1)
    v.mul_(beta2).addcmul_(g, g, value=1 - beta2)
    mh = m / (1 - beta1 ** step)
    vh = v / (1 - beta2 ** step)
    p32.mul_(1 - lr * wd).addcdiv_(mh, vh.sqrt().add_(eps), value=-lr)
