"""Each sm_100a kernel against the fp32 PyTorch definition of the same op."""

import math

import pytest
import torch

from lumenrl_b200 import ops
from lumenrl_b200.ops import reference as ref

pytestmark = pytest.mark.gpu


def close(a, b, atol, rtol=0.0):
    a, b = a.float().cpu(), b.float().cpu()
    err = (a - b).abs().max().item()
    tol = atol + rtol * b.abs().max().item()
    assert err <= tol, f"max abs err {err} > {tol}"


@pytest.mark.parametrize("T,H", [(1, 256), (37, 4096), (129, 1000 * 8), (1, 32768), (400, 32768)])
def test_rmsnorm_fwd_bwd(cuda, T, H):
    """Includes the launch-shape edges: one row, more rows than two per SM
    (the many-rows branch), and the widest rows (32768, 1024 threads)."""
    torch.manual_seed(0)
    x = torch.randn(T, H, device=cuda, dtype=torch.bfloat16, requires_grad=True)
    w = (1 + 0.1 * torch.randn(H, device=cuda)).to(torch.bfloat16)
    wp = torch.nn.Parameter(w.clone())
    wp.main_grad = torch.zeros(H, device=cuda)
    y = ops.rmsnorm(x, wp, 1e-6)
    xr = x.detach().float().requires_grad_(True)
    wr = w.float().requires_grad_(True)
    yr = xr * torch.rsqrt(xr.pow(2).mean(-1, keepdim=True) + 1e-6) * wr
    close(y, yr, 2e-2, 1e-2)
    g = torch.randn_like(yr)
    y.backward(g.to(torch.bfloat16))
    yr.backward(g)
    close(x.grad, xr.grad, 3e-2, 2e-2)
    close(wp.main_grad, wr.grad, 0.5, 1e-2)


@pytest.mark.parametrize("T,H", [(64, 4096), (1, 16384), (400, 16384)])
def test_add_rmsnorm(cuda, T, H):
    torch.manual_seed(0)
    x = torch.randn(T, H, device=cuda, dtype=torch.bfloat16)
    r = torch.randn(T, H, device=cuda, dtype=torch.bfloat16)
    w = torch.randn(H, device=cuda).to(torch.bfloat16)
    with torch.no_grad():
        y, s = ops.add_rmsnorm(x, r, w, 1e-6)
    s_ref = (x + r)
    close(s, s_ref, 0.0)
    close(y, ref.rmsnorm(s_ref.float(), w.float(), 1e-6), 3e-2, 1e-2)


def test_add_rmsnorm_rejects_rows_wider_than_16384(cuda):
    x = torch.randn(4, 16392, device=cuda, dtype=torch.bfloat16)
    w = torch.ones(16392, device=cuda, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError):
        with torch.no_grad():
            ops.add_rmsnorm(x, x.clone(), w, 1e-6)


def test_add_rmsnorm_fwd_bwd(cuda):
    """Fused add + RMSNorm with autograd (both outputs carry gradient; the
    sum's gradient is added inside the RMSNorm backward kernel) against fp32."""
    torch.manual_seed(3)
    T, H = 333, 4096
    x = torch.randn(T, H, device=cuda, dtype=torch.bfloat16, requires_grad=True)
    r = torch.randn(T, H, device=cuda, dtype=torch.bfloat16, requires_grad=True)
    wp = torch.nn.Parameter((1 + 0.1 * torch.randn(H, device=cuda)).to(torch.bfloat16))
    wp.main_grad = torch.zeros(H, device=cuda)
    y, s = ops.add_rmsnorm(x, r, wp, 1e-6)
    gy, gs = torch.randn(T, H, device=cuda), torch.randn(T, H, device=cuda)
    (y.float() * gy + s.float() * gs).sum().backward()
    xr, rr = x.detach().float().requires_grad_(True), r.detach().float().requires_grad_(True)
    wr = wp.detach().float().requires_grad_(True)
    sr = xr + rr
    yr = sr * torch.rsqrt(sr.pow(2).mean(-1, keepdim=True) + 1e-6) * wr
    (yr * gy + sr * gs).sum().backward()
    close(y, yr, 3e-2, 1e-2)
    close(s, sr, 2e-2, 1e-2)
    close(x.grad, xr.grad, 5e-2, 2e-2)
    close(r.grad, rr.grad, 5e-2, 2e-2)
    close(wp.main_grad, wr.grad, 1.0, 1e-2)


@pytest.mark.parametrize("hd,nh,nkv,norm", [(128, 32, 8, True), (64, 4, 2, False), (128, 4, 4, True)])
def test_qk_norm_rope(cuda, hd, nh, nkv, norm):
    torch.manual_seed(0)
    T = 77
    qkv = torch.randn(T, (nh + 2 * nkv) * hd, device=cuda, dtype=torch.bfloat16, requires_grad=True)
    pos = torch.randint(0, 4000, (T,), device=cuda)
    inv = ops.inv_freq_table(hd, 1e6, None, cuda)
    qw = torch.nn.Parameter((1 + 0.1 * torch.randn(hd, device=cuda)).to(torch.bfloat16)) if norm else None
    kw = torch.nn.Parameter((1 + 0.1 * torch.randn(hd, device=cuda)).to(torch.bfloat16)) if norm else None
    if norm:
        qw.main_grad = torch.zeros(hd, device=cuda)
        kw.main_grad = torch.zeros(hd, device=cuda)
    q, k, v = ops.qk_norm_rope(qkv, qw, kw, pos, inv, nh, nkv, hd, 1e-6)
    # fp32 reference with autograd
    xr = qkv.detach().float().requires_grad_(True)
    qwr = qw.detach().float().requires_grad_(True) if norm else None
    kwr = kw.detach().float().requires_grad_(True) if norm else None
    ang = pos.float().unsqueeze(-1) * inv.unsqueeze(0)
    cos, sin = ang.cos(), ang.sin()

    def nrm(t, w):
        return t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + 1e-6) * w if w is not None else t

    def rope(t):
        d = t.shape[-1] // 2
        c, s = cos.unsqueeze(1), sin.unsqueeze(1)
        return torch.cat([t[..., :d] * c - t[..., d:] * s, t[..., d:] * c + t[..., :d] * s], -1)
    qr = rope(nrm(xr[:, : nh * hd].view(T, nh, hd), qwr))
    kr = rope(nrm(xr[:, nh * hd:(nh + nkv) * hd].view(T, nkv, hd), kwr))
    vr = xr[:, (nh + nkv) * hd:].view(T, nkv, hd)
    close(q, qr, 3e-2, 1e-2)
    close(k, kr, 3e-2, 1e-2)
    close(v, vr, 0.0)
    gq, gk, gv = torch.randn_like(qr), torch.randn_like(kr), torch.randn_like(vr)
    torch.autograd.backward([q, k, v], [gq.bfloat16(), gk.bfloat16(), gv.bfloat16()])
    torch.autograd.backward([qr, kr, vr], [gq, gk, gv])
    close(qkv.grad, xr.grad, 5e-2, 2e-2)
    if norm:
        close(qw.main_grad, qwr.grad, 0.5, 2e-2)
        close(kw.main_grad, kwr.grad, 0.5, 2e-2)


def test_swiglu(cuda):
    torch.manual_seed(0)
    gu = torch.randn(33, 2 * 688, device=cuda, dtype=torch.bfloat16, requires_grad=True)
    h = ops.swiglu(gu)
    gr = gu.detach().float().requires_grad_(True)
    hr = torch.nn.functional.silu(gr[:, :688]) * gr[:, 688:]
    close(h, hr, 3e-2, 1e-2)
    g = torch.randn_like(hr)
    h.backward(g.bfloat16())
    hr.backward(g)
    close(gu.grad, gr.grad, 5e-2, 1e-2)


@pytest.mark.parametrize("V,temp", [(2048, 1.0), (151936, 0.7)])
def test_token_logprob_fwd_bwd(cuda, V, temp):
    torch.manual_seed(0)
    N, H = 70, 256
    hidden = (0.5 * torch.randn(N, H, device=cuda)).to(torch.bfloat16).requires_grad_(True)
    W = torch.nn.Parameter((0.05 * torch.randn(V, H, device=cuda)).to(torch.bfloat16))
    W.main_grad = torch.zeros(V, H, device=cuda)
    tgt = torch.randint(0, V, (N,), device=cuda)
    lp, ent = ops.token_logprob(hidden, W, tgt, temperature=temp, chunk=32)
    hr = hidden.detach().float().requires_grad_(True)
    Wr = W.detach().float().requires_grad_(True)
    z = (hr @ Wr.t()) / temp
    lpr = z.log_softmax(-1).gather(-1, tgt.unsqueeze(-1)).squeeze(-1)
    p = z.softmax(-1)
    entr = -(p * z.log_softmax(-1)).sum(-1)
    close(lp, lpr, 2e-2, 1e-3)
    close(ent, entr, 2e-2, 1e-3)
    g1, g2 = torch.randn(N, device=cuda), torch.randn(N, device=cuda)
    torch.autograd.backward([lp, ent], [g1, g2])
    torch.autograd.backward([lpr, entr], [g1, g2])
    close(hidden.grad, hr.grad, 2e-2, 2e-2)
    close(W.main_grad, Wr.grad, 2e-2, 2e-2)


def test_group_advantage(cuda):
    r = torch.randint(0, 2, (64,), device=cuda).float()
    for unb in (False, True):
        close(ops.group_advantage(r, 8, unb), ref.group_advantage(r.cpu(), 8, unb, 1e-8), 1e-5)


@pytest.mark.parametrize("clip_c,with_w", [(0.0, False), (3.0, True)])
def test_ppo_clip_loss(cuda, clip_c, with_w):
    torch.manual_seed(0)
    n = 5000
    old = -torch.rand(n, device=cuda) * 3
    logp = (old + 0.3 * torch.randn(n, device=cuda)).requires_grad_(True)
    adv = torch.randn(n, device=cuda)
    mask = (torch.rand(n, device=cuda) > 0.2).float()
    w = torch.rand(n, device=cuda) * 2 if with_w else None
    loss = ops.ppo_clip_loss(logp, old, adv, mask, 0.2, 0.28, clip_c, w, denom=1234.0)
    lr = logp.detach().clone().requires_grad_(True)
    loss_r = ref.ppo_clip_token_loss(lr, old, adv, mask, 0.2, 0.28, clip_c, w, 1234.0)
    close(loss, loss_r, 1e-4, 1e-5)
    loss.backward()
    loss_r.backward()
    close(logp.grad, lr.grad, 1e-6, 1e-5)


def test_adamw_matches_reference(cuda):
    torch.manual_seed(0)
    n = 4096 * 3
    p = torch.randn(n, device=cuda)
    g = torch.randn(n, device=cuda)
    m, v = torch.zeros(n, device=cuda), torch.zeros(n, device=cuda)
    w16 = torch.empty(n, device=cuda, dtype=torch.bfloat16)
    pr, mr, vr = p.cpu().clone(), m.cpu().clone(), v.cpu().clone()
    from lumenrl_b200.ops.ext import ext
    for step in (1, 2, 3):
        ext().adamw_step(p, g, m, v, w16, 1e-3, 0.9, 0.95, 1e-8, 0.01, step, 0.5)
        ref.adamw_reference(pr, g.cpu(), mr, vr, 1e-3, 0.9, 0.95, 1e-8, 0.01, step, 0.5)
    close(p, pr, 1e-5, 1e-5)
    close(w16, pr, 1e-2, 4e-3)
    close(ext().sumsq(g), (g.double() ** 2).sum(), 1e-1, 1e-5)


@pytest.mark.parametrize("kv_dtype", [torch.bfloat16, torch.float8_e4m3fn])
@pytest.mark.parametrize("B,Hq,Hk,bs,maxlen", [(3, 32, 8, 64, 700), (64, 32, 8, 64, 1536), (5, 4, 2, 16, 90)])
def test_paged_decode_attention(cuda, kv_dtype, B, Hq, Hk, bs, maxlen):
    torch.manual_seed(0)
    D = 128
    lens = torch.randint(1, maxlen + 1, (B,), device=cuda, dtype=torch.int32)
    lens[0] = maxlen
    mb = (maxlen + bs - 1) // bs
    nblocks = B * mb + 3
    perm = torch.randperm(nblocks - 1, device=cuda)[: B * mb] + 1
    bt = perm.view(B, mb).to(torch.int32)
    kc = torch.randn(nblocks, bs, Hk, D, device=cuda).to(kv_dtype)
    vc = torch.randn(nblocks, bs, Hk, D, device=cuda).to(kv_dtype)
    q = torch.randn(B, Hq, D, device=cuda, dtype=torch.bfloat16)
    ks, vs = (0.5, 2.0) if kv_dtype != torch.bfloat16 else (1.0, 1.0)
    out = ops.paged_decode_attention(q, kc, vc, bt, lens, 1 / math.sqrt(D), ks, vs, maxlen)
    out_r = ref.paged_decode_attention(q.cpu(), kc.float().cpu() * ks, vc.float().cpu() * vs, bt.cpu(), lens.cpu(),
                                       1 / math.sqrt(D))
    close(out, out_r, 2e-2, 2e-2)


@pytest.mark.parametrize("kv_dtype", [torch.bfloat16, torch.float8_e4m3fn])
@pytest.mark.parametrize("n,Hq,Hk,bs,plen,maxnew", [(8, 32, 8, 16, 512, 300), (4, 32, 8, 16, 100, 70),
                                                    (16, 16, 4, 16, 200, 129), (8, 32, 8, 16, 8, 64),
                                                    (2, 8, 1, 32, 96, 33)])
def test_paged_decode_attention_shared_prefix(cuda, kv_dtype, n, Hq, Hk, bs, plen, maxnew):
    """Rows of a group share the prompt's whole KV blocks; the shared-prefix
    kernel must equal the fp32 reference of plain paged attention."""
    torch.manual_seed(1)
    D, P = 128, 3
    B = P * n
    full = plen // bs                         # shared whole blocks
    need = (plen + maxnew + bs - 1) // bs
    nblocks = 1 + P * full + B * (need - full) + 2
    perm = (torch.randperm(nblocks - 1) + 1).tolist()
    bt = torch.zeros(B, need, dtype=torch.int32)
    for i in range(P):
        shared = [perm.pop() for _ in range(full)]
        for j in range(n):
            bt[i * n + j, :full] = torch.tensor(shared, dtype=torch.int32)
            bt[i * n + j, full:] = torch.tensor([perm.pop() for _ in range(need - full)], dtype=torch.int32)
    bt = bt.to(cuda)
    lens = (plen + torch.randint(1, maxnew + 1, (B,))).to(torch.int32)
    lens[0] = plen + maxnew
    lens = lens.to(cuda)
    prefix = torch.full((B,), full * bs, dtype=torch.int32, device=cuda)
    kc = torch.randn(nblocks, bs, Hk, D, device=cuda).to(kv_dtype)
    vc = torch.randn(nblocks, bs, Hk, D, device=cuda).to(kv_dtype)
    q = torch.randn(B, Hq, D, device=cuda, dtype=torch.bfloat16)
    ks, vs = (0.5, 2.0) if kv_dtype != torch.bfloat16 else (1.0, 1.0)
    grp = ops.shared_prefix_group(n, Hq // Hk)
    out = ops.paged_decode_attention_shared(q, kc, vc, bt, lens, prefix, grp, 1 / math.sqrt(D), ks, vs,
                                            full * bs, maxnew + bs)
    out_r = ref.paged_decode_attention(q.cpu(), kc.float().cpu() * ks, vc.float().cpu() * vs, bt.cpu(), lens.cpu(),
                                       1 / math.sqrt(D))
    close(out, out_r, 2e-2, 2e-2)
    plain = ops.paged_decode_attention(q, kc, vc, bt, lens, 1 / math.sqrt(D), ks, vs, plen + maxnew)
    close(out, plain, 2e-2, 2e-2)


def test_kv_append_roundtrip(cuda):
    T, Hk, D, bs = 50, 8, 128, 16
    kc = torch.zeros(10, bs, Hk, D, device=cuda, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    k = torch.randn(T, Hk, D, device=cuda, dtype=torch.bfloat16)
    v = torch.randn(T, Hk, D, device=cuda, dtype=torch.bfloat16)
    slots = torch.randperm(10 * bs, device=cuda)[:T]
    ops.kv_cache_append(k, v, kc, vc, slots)
    close(kc.view(-1, Hk, D)[slots], k, 0.0)
    close(vc.view(-1, Hk, D)[slots], v, 0.0)


def test_sampler_distribution(cuda):
    torch.manual_seed(0)
    V = 50
    logits = torch.randn(1, V, device=cuda).repeat(4096, 1)
    seeds = torch.arange(4096, device=cuda)
    step = torch.zeros(1, dtype=torch.long, device=cuda)
    tok, lp = ops.sample_tokens_device(logits, 1.0, 1.0, seeds, step)
    p = torch.softmax(logits[0].float(), -1)
    freq = torch.bincount(tok, minlength=V).float() / 4096
    assert (freq - p).abs().max().item() < 0.03
    close(lp, torch.log(p)[tok], 1e-4)
    # same seed + step -> same draw; top-p keeps only the nucleus
    tok2, _ = ops.sample_tokens_device(logits, 1.0, 1.0, seeds, step)
    assert torch.equal(tok, tok2)
    tk, _ = ops.sample_tokens_device(logits, 1.0, 0.5, seeds, step)
    srt, idx = torch.sort(p, descending=True)
    keep = set(idx[: int((torch.cumsum(srt, 0) < 0.5).sum()) + 1].tolist())
    assert set(tk.tolist()) <= keep


def test_sampler_split_rows_large_vocab(cuda):
    torch.manual_seed(0)
    V = 151936
    base = torch.full((V,), -30.0, device=cuda)
    hot = torch.randint(0, V, (40,), device=cuda).unique()
    base[hot] = torch.randn(hot.numel(), device=cuda)
    logits = base.to(torch.bfloat16).unsqueeze(0).repeat(4096, 1)
    tok, lp = ops.sample_tokens_device(logits, 1.0, 1.0, torch.arange(4096, device=cuda),
                                      torch.zeros(1, dtype=torch.long, device=cuda))
    p = torch.softmax(logits[0].float(), -1)
    freq = torch.bincount(tok, minlength=V).float() / 4096
    assert (freq - p).abs().max().item() < 0.03
    close(lp, torch.log(p)[tok], 1e-3)


def test_qk_norm_rope_cache_write(cuda):
    torch.manual_seed(0)
    T, nh, nkv, hd, bs = 9, 8, 2, 128, 16
    qkv = torch.randn(T, (nh + 2 * nkv) * hd, device=cuda, dtype=torch.bfloat16)
    pos = torch.arange(T, device=cuda) + 5
    inv = ops.inv_freq_table(hd, 1e6, None, cuda)
    qw = (1 + 0.1 * torch.randn(hd, device=cuda)).to(torch.bfloat16)
    kw = (1 + 0.1 * torch.randn(hd, device=cuda)).to(torch.bfloat16)
    kc = torch.zeros(4, bs, nkv, hd, device=cuda, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    slots = torch.randperm(4 * bs, device=cuda)[:T]
    q, k, v = ops.qk_norm_rope_cache(qkv, qw, kw, pos, inv, nh, nkv, hd, 1e-6, kc, vc, slots)
    q2, k2, v2 = ops.qk_norm_rope(qkv, qw, kw, pos, inv, nh, nkv, hd, 1e-6)
    close(q, q2, 0.0)
    close(kc.view(-1, nkv, hd)[slots], k2, 0.0)
    close(vc.view(-1, nkv, hd)[slots], v2, 0.0)


def test_attention_varlen_fwd_bwd(cuda):
    """Packed causal GQA attention (one varlen flash call) against an fp32
    per-sequence reference, forward and backward."""
    torch.manual_seed(0)
    lens = [37, 200, 1, 511]
    T, Hq, Hk, D = sum(lens), 8, 2, 128
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32, device=cuda)
    q = torch.randn(T, Hq, D, device=cuda).to(torch.bfloat16).requires_grad_(True)
    k = torch.randn(T, Hk, D, device=cuda).to(torch.bfloat16).requires_grad_(True)
    v = torch.randn(T, Hk, D, device=cuda).to(torch.bfloat16).requires_grad_(True)
    do = torch.randn(T, Hq, D, device=cuda).to(torch.bfloat16)
    o = ops.attention_varlen(q, k, v, cu, max(lens), causal=True, scale=D ** -0.5)
    o.backward(do)
    qr, kr, vr = (t.detach().float().requires_grad_(True) for t in (q, k, v))
    outs = []
    a = 0
    for n in lens:
        qi, ki, vi = qr[a:a + n].transpose(0, 1), kr[a:a + n].transpose(0, 1), vr[a:a + n].transpose(0, 1)
        ki, vi = ki.repeat_interleave(Hq // Hk, 0), vi.repeat_interleave(Hq // Hk, 0)
        s = (qi @ ki.transpose(-1, -2)) * D ** -0.5
        s = s.masked_fill(torch.ones(n, n, dtype=torch.bool, device=cuda).triu(1), float("-inf"))
        outs.append((torch.softmax(s, -1) @ vi).transpose(0, 1))
        a += n
    ref = torch.cat(outs)
    ref.backward(do.float())
    close(o, ref, 2e-2, 2e-2)
    for g, r in ((q.grad, qr.grad), (k.grad, kr.grad), (v.grad, vr.grad)):
        assert ((g.float() - r).abs().max() / r.abs().max()).item() < 2e-2


@pytest.mark.parametrize("shared", [False, True])
@pytest.mark.parametrize("n,Hq,Hk,plen,maxnew", [(8, 32, 8, 512, 300), (4, 32, 8, 130, 70), (16, 16, 4, 64, 129),
                                                 (2, 8, 1, 0, 65)])
def test_decode_attention_tma_pages(cuda, monkeypatch, shared, n, Hq, Hk, plen, maxnew):
    """TMA-fed decode attention (64-token pages streamed by a producer warp)
    against the fp32 reference, per-row and shared-prefix."""
    monkeypatch.setattr(ops, "DECODE_ATTN", "tma")
    torch.manual_seed(2)
    D, bs, P = 128, 64, 3
    B = P * n
    full = plen // bs
    need = (plen + maxnew + bs - 1) // bs
    nblocks = 1 + P * full + B * (need - full) + 2
    perm = (torch.randperm(nblocks - 1) + 1).tolist()
    bt = torch.zeros(B, need + 1, dtype=torch.int32)
    for i in range(P):
        sh = [perm.pop() for _ in range(full)]
        for j in range(n):
            bt[i * n + j, :full] = torch.tensor(sh, dtype=torch.int32)
            bt[i * n + j, full:need] = torch.tensor([perm.pop() for _ in range(need - full)], dtype=torch.int32)
    bt = bt.to(cuda)
    lens = (plen + torch.randint(1, maxnew + 1, (B,))).to(torch.int32)
    lens[0] = plen + maxnew
    lens = lens.to(cuda)
    kc = torch.randn(nblocks, bs, Hk, D, device=cuda).to(torch.bfloat16)
    vc = torch.randn(nblocks, bs, Hk, D, device=cuda).to(torch.bfloat16)
    q = torch.randn(B, Hq, D, device=cuda, dtype=torch.bfloat16)
    sc = 1 / math.sqrt(D)
    if shared:
        prefix = torch.full((B,), full * bs, dtype=torch.int32, device=cuda)
        out = ops.paged_decode_attention_shared(q, kc, vc, bt, lens, prefix, ops.shared_prefix_group(n, Hq // Hk),
                                                sc, 1.0, 1.0, full * bs, maxnew + bs)
    else:
        out = ops.paged_decode_attention(q, kc, vc, bt, lens, sc, 1.0, 1.0, plen + maxnew)
    torch.cuda.synchronize()
    from lumenrl_b200.ops.ext import ext
    assert ext().decode_tma_status() == 0
    out_r = ref.paged_decode_attention(q.cpu(), kc.float().cpu(), vc.float().cpu(), bt.cpu(), lens.cpu(), sc)
    close(out, out_r, 2e-2, 2e-2)


def _causal_ref(q, k, v, lens, scale, causal=True):
    """fp32 per-sequence (causal) GQA attention: output [T, Hq, D], LSE [Hq, T]."""
    Hq, Hk = q.shape[1], k.shape[1]
    outs, lses, a = [], [], 0
    for n in lens:
        qi, ki, vi = q[a:a + n].transpose(0, 1), k[a:a + n].transpose(0, 1), v[a:a + n].transpose(0, 1)
        ki, vi = ki.repeat_interleave(Hq // Hk, 0), vi.repeat_interleave(Hq // Hk, 0)
        s = (qi @ ki.transpose(-1, -2)) * scale
        if causal:
            s = s.masked_fill(torch.ones(n, n, dtype=torch.bool, device=q.device).triu(1), float("-inf"))
        lses.append(torch.logsumexp(s, -1))
        outs.append((torch.softmax(s, -1) @ vi).transpose(0, 1))
        a += n
    return torch.cat(outs), torch.cat(lses, 1)


@pytest.mark.parametrize("variant", [0, 1, 2, 3, 4])
@pytest.mark.parametrize("lens", [[128], [1, 100, 129, 300], [513, 7, 256, 1024]])
def test_fa_fwd_tcgen05(cuda, lens, variant):
    """tcgen05 flash-attention forward (ragged packed sequences, GQA 4:1) in
    each softmax variant against the fp32 reference: output and natural-log
    LSE."""
    from lumenrl_b200.ops.ext import ext
    torch.manual_seed(0)
    T, Hq, Hk, D = sum(lens), 8, 2, 128
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32, device=cuda)
    q = torch.randn(T, Hq, D, device=cuda).to(torch.bfloat16)
    k = torch.randn(T, Hk, D, device=cuda).to(torch.bfloat16)
    v = torch.randn(T, Hk, D, device=cuda).to(torch.bfloat16)
    out, lse = ext().fa_fwd(q, k, v, cu, max(lens), D ** -0.5, variant)
    assert ext().fa_fwd_status() == 0
    ro, rl = _causal_ref(q.float(), k.float(), v.float(), lens, D ** -0.5)
    close(out, ro, 2e-2, 2e-2)
    close(lse, rl, 1e-2, 1e-3)


@pytest.mark.parametrize("mode", ["tc", "fa2", "tc+tc"])
def test_fa_fwd_bwd_modes(cuda, monkeypatch, mode):
    """Training attention with the tcgen05 forward (gradients through the
    library backward fed with its output and LSE) and with the library
    forward."""
    from lumenrl_b200.ops import attention
    monkeypatch.setattr(attention, "TRAIN_ATTN", mode.split("+")[0])
    monkeypatch.setattr(attention, "TRAIN_ATTN_BWD", "tc" if mode == "tc+tc" else "fa2")
    torch.manual_seed(1)
    lens = [37, 200, 1, 511]
    T, Hq, Hk, D = sum(lens), 8, 2, 128
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32, device=cuda)
    q = torch.randn(T, Hq, D, device=cuda).to(torch.bfloat16).requires_grad_(True)
    k = torch.randn(T, Hk, D, device=cuda).to(torch.bfloat16).requires_grad_(True)
    v = torch.randn(T, Hk, D, device=cuda).to(torch.bfloat16).requires_grad_(True)
    do = torch.randn(T, Hq, D, device=cuda).to(torch.bfloat16)
    o = ops.attention_varlen(q, k, v, cu, max(lens), causal=True, scale=D ** -0.5)
    o.backward(do)
    qr, kr, vr = (t.detach().float().requires_grad_(True) for t in (q, k, v))
    ro, _ = _causal_ref(qr, kr, vr, lens, D ** -0.5)
    ro.backward(do.float())
    close(o, ro, 2e-2, 2e-2)
    for g, r in ((q.grad, qr.grad), (k.grad, kr.grad), (v.grad, vr.grad)):
        assert ((g.float() - r).abs().max() / r.abs().max()).item() < 2e-2


@pytest.mark.parametrize("variant", [0, 1])
@pytest.mark.parametrize("lens", [[128], [1, 100, 129, 300], [513, 7, 256, 1024]])
def test_fa_bwd_tcgen05(cuda, lens, variant):
    """tcgen05 flash-attention backward (dQ kernel + dK/dV kernel, GQA 4:1,
    ragged packed sequences) against fp32 autograd of the causal reference."""
    from lumenrl_b200.ops.ext import ext
    torch.manual_seed(2)
    T, Hq, Hk, D = sum(lens), 8, 2, 128
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32, device=cuda)
    q = torch.randn(T, Hq, D, device=cuda).to(torch.bfloat16)
    k = torch.randn(T, Hk, D, device=cuda).to(torch.bfloat16)
    v = torch.randn(T, Hk, D, device=cuda).to(torch.bfloat16)
    do = torch.randn(T, Hq, D, device=cuda).to(torch.bfloat16)
    out, lse = ext().fa_fwd(q, k, v, cu, max(lens), D ** -0.5)
    dq, dk, dv = ext().fa_bwd(do, q, k, v, out, lse, cu, max(lens), D ** -0.5, variant=variant)
    assert ext().fa_bwd_status() == 0
    qr, kr, vr = (t.float().requires_grad_(True) for t in (q, k, v))
    ro, _ = _causal_ref(qr, kr, vr, lens, D ** -0.5)
    ro.backward(do.float())
    for g, r in ((dq, qr.grad), (dk, kr.grad), (dv, vr.grad)):
        assert ((g.float() - r).abs().max() / r.abs().max()).item() < 2e-2


@pytest.mark.parametrize("lens", [[128], [1, 100, 129, 300], [513, 7, 256, 1024]])
def test_fa_noncausal_fwd_bwd_tcgen05(cuda, lens):
    """The unmasked mode of the tcgen05 flash kernels (ring-attention blocks
    off the diagonal): forward, LSE and all three gradients against fp32."""
    from lumenrl_b200.ops.ext import ext
    torch.manual_seed(4)
    T, Hq, Hk, D = sum(lens), 8, 2, 128
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32, device=cuda)
    q = torch.randn(T, Hq, D, device=cuda).to(torch.bfloat16)
    k = torch.randn(T, Hk, D, device=cuda).to(torch.bfloat16)
    v = torch.randn(T, Hk, D, device=cuda).to(torch.bfloat16)
    do = torch.randn(T, Hq, D, device=cuda).to(torch.bfloat16)
    out, lse = ext().fa_fwd(q, k, v, cu, max(lens), D ** -0.5, causal=False)
    dq, dk, dv = ext().fa_bwd(do, q, k, v, out, lse, cu, max(lens), D ** -0.5, causal=False)
    assert ext().fa_fwd_status() == 0 and ext().fa_bwd_status() == 0
    qr, kr, vr = (t.float().requires_grad_(True) for t in (q, k, v))
    ro, rl = _causal_ref(qr, kr, vr, lens, D ** -0.5, causal=False)
    close(out, ro.detach(), 2e-2, 2e-2)
    close(lse, rl.detach(), 1e-2, 1e-3)
    ro.backward(do.float())
    for g, r in ((dq, qr.grad), (dk, kr.grad), (dv, vr.grad)):
        assert ((g.float() - r).abs().max() / r.abs().max()).item() < 2e-2


def test_ring_attention_blocks_on_tcgen05(cuda):
    """Context parallelism emulated on one GPU: the zigzag ring of cp = 2
    ranks run as its four (query chunk, key chunk) blocks through the block
    functions ring attention uses, merged by LSE, against full causal
    attention of the whole sequence; gradients through the global LSE."""
    from lumenrl_b200.parallel import context_parallel as cpm
    torch.manual_seed(5)
    B, H, Hk, S, D, cp = 2, 8, 2, 1024, 128, 2
    q = torch.randn(B, H, S, D, device=cuda).to(torch.bfloat16)
    k = torch.randn(B, Hk, S, D, device=cuda).to(torch.bfloat16)
    v = torch.randn(B, Hk, S, D, device=cuda).to(torch.bfloat16)
    c = S // (2 * cp)
    chunks = lambda x, i: x[:, :, i * c:(i + 1) * c].contiguous()  # noqa: E731
    outs = {}
    for qi in range(2 * cp):
        o = lse = None
        for ki in range(qi + 1):
            ob, lb = cpm._block_fwd(chunks(q, qi), chunks(k, ki), chunks(v, ki), ki == qi, D ** -0.5)
            o, lse = cpm._merge(o, lse, ob, lb)
        outs[qi] = (o, lse)
    full = torch.cat([outs[i][0] for i in range(2 * cp)], 2)
    ref = torch.nn.functional.scaled_dot_product_attention(
        q.float(), k.float().repeat_interleave(H // Hk, 1), v.float().repeat_interleave(H // Hk, 1),
        is_causal=True, scale=D ** -0.5)
    close(full, ref, 2e-2, 2e-2)
    # backward of one off-diagonal block from the merged output / LSE
    do = torch.randn(B, H, c, D, device=cuda).to(torch.bfloat16)
    o3, l3 = outs[3]
    dq, dk, dv = cpm._block_bwd(do, chunks(q, 3), chunks(k, 1), chunks(v, 1), o3.to(torch.bfloat16), l3, False,
                                D ** -0.5)
    qr, kr, vr = (chunks(t, i).float().requires_grad_(True) for t, i in ((q, 3), (k, 1), (v, 1)))
    s = (qr @ kr.repeat_interleave(H // Hk, 1).transpose(-1, -2)) * D ** -0.5
    p = torch.exp(s - l3.unsqueeze(-1))
    (p @ vr.repeat_interleave(H // Hk, 1)).backward(do.float())
    # dq of the block alone omits the softmax-normaliser term carried by D = rowsum(dO o O):
    # compare dv (linear in P) exactly, dq/dk through the full formula
    assert ((dv - vr.grad).abs().max() / vr.grad.abs().max()).item() < 2e-2
    D_ = (do.float() * o3.float()).sum(-1, keepdim=True)
    dp = do.float() @ vr.detach().repeat_interleave(H // Hk, 1).transpose(-1, -2)
    ds = p.detach() * (dp - D_) * D ** -0.5
    dq_ref = ds @ kr.detach().repeat_interleave(H // Hk, 1)
    assert ((dq - dq_ref).abs().max() / dq_ref.abs().max()).item() < 2e-2
