"""Eagle3 TTT attention and forward-KL kernels against fp32 PyTorch references."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a GPU", allow_module_level=True)

from lumenrl_b200.models.eagle3 import Eagle3Model, cached_tree_attention  # noqa: E402
from lumenrl_b200.ops.eagle import forward_kl, ttt_attention  # noqa: E402


def _rel(a, b):
    return float((a.float() - b.float()).abs().max() / b.float().abs().max().clamp_min(1e-6))


@pytest.mark.parametrize("nd", [0, 1, 3, 6])
def test_ttt_attention_matches_tree_attention(nd):
    torch.manual_seed(nd)
    lens = [100, 257, 64, 1]
    T, H, KVH, D = sum(lens), 8, 2, 128
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32, device="cuda")
    scale = 1 / math.sqrt(D)

    def r(*s):
        return (torch.randn(*s, device="cuda") * 1.5).to(torch.bfloat16)
    q = r(T, H, D)
    cache = [(r(T, KVH, D), r(T, KVH, D)) for _ in range(nd + 1)]
    dout = r(T, H, D)
    # kernels
    qk = q.clone().requires_grad_()
    ck = [(k.clone().requires_grad_(), v.clone().requires_grad_()) for k, v in cache]
    out = ttt_attention(qk, ck, cu, max(lens), scale)
    out.backward(dout)
    # fp32 reference on the same bf16 inputs
    qr = q.float().requires_grad_()
    cr = [(k.float().requires_grad_(), v.float().requires_grad_()) for k, v in cache]
    ref = cached_tree_attention(qr, cr, cu, scale)
    ref.backward(dout.float())
    assert _rel(out, ref) < 2e-2
    assert _rel(qk.grad, qr.grad) < 3e-2
    for (kk, vk), (kr, vr) in zip(ck, cr):
        assert _rel(kk.grad, kr.grad) < 3e-2
        assert _rel(vk.grad, vr.grad) < 3e-2


def _fkl_ref(dh, wd, th, wt):
    zt = (th.float() @ wt.float().t()).to(torch.bfloat16).double()
    zd = dh.float() @ wd.float().t()
    lp = torch.log_softmax(zt, -1)
    lq = torch.log_softmax(zd.double(), -1)
    kl = (lp.exp() * (lp - lq)).sum(-1)
    hit = (zd.argmax(-1) == zt.argmax(-1)).float()
    return kl, hit


def test_forward_kl_matches_reference():
    torch.manual_seed(1)
    n, Hd, V = 700, 256, 2048
    dh = (torch.randn(n, Hd, device="cuda") * 0.5).to(torch.bfloat16)
    th = (torch.randn(n, Hd, device="cuda") * 0.5).to(torch.bfloat16)
    wd = (torch.randn(V, Hd, device="cuda") * 0.1).to(torch.bfloat16)
    wt = (torch.randn(V, Hd, device="cuda") * 0.1).to(torch.bfloat16)
    dk = dh.clone().requires_grad_()
    wk = wd.clone().requires_grad_()
    kl, hit = forward_kl(dk, wk, th, wt, chunk=256)
    g = torch.rand(n, device="cuda")
    (kl * g).sum().backward()
    dr = dh.float().requires_grad_()
    wr = wd.float().requires_grad_()
    klr, hitr = _fkl_ref(dr, wr, th, wt)
    (klr * g.double()).sum().backward()
    assert float((kl.double() - klr).abs().max()) < 5e-3 * max(1.0, float(klr.abs().max()))
    assert float((hit - hitr).abs().mean()) < 0.02      # arg-max ties under bf16 rounding
    assert _rel(dk.grad, dr.grad) < 3e-2
    assert _rel(wk.grad, wr.grad) < 3e-2


def test_eagle3_model_kernels_match_torch_path():
    torch.manual_seed(0)
    Hd, V, Vd = 512, 4096, 1024
    m = Eagle3Model(Hd, V, Vd, 4, 2, 128, ffn=1024, length=3).cuda()
    m16 = Eagle3Model(Hd, V, Vd, 4, 2, 128, ffn=1024, length=3).cuda()
    m16.load_state_dict(m.state_dict())
    m16 = m16.to(torch.bfloat16)
    lens = [96, 160]
    T = sum(lens)
    cu = torch.tensor([0, 96, 256], dtype=torch.int32, device="cuda")
    ids = torch.randint(0, V, (T,), device="cuda")
    aux = (torch.randn(T, 3 * Hd, device="cuda") * 0.5).to(torch.bfloat16)
    tgt = (torch.randn(T, Hd, device="cuda") * 0.5).to(torch.bfloat16)
    emb = (torch.randn(V, Hd, device="cuda") * 0.02).to(torch.bfloat16)
    head = (torch.randn(V, Hd, device="cuda") * 0.05).to(torch.bfloat16)
    mask = torch.ones(T, device="cuda")
    out16 = m16(ids, aux, tgt, emb, head, cu, mask)
    out16["loss"].backward()
    # fp32 parameters take the PyTorch path on the same (bf16-rounded) weights
    ref = Eagle3Model(Hd, V, Vd, 4, 2, 128, ffn=1024, length=3).cuda()
    ref.load_state_dict({k: (v.float() if v.is_floating_point() else v) for k, v in m16.state_dict().items()})
    outr = ref(ids, aux.float(), tgt.float(), emb.float(), head.float(), cu, mask)
    assert abs(float(out16["loss"]) - float(outr["loss"])) < 3e-2 * max(1.0, abs(float(outr["loss"])))
    for a, b in zip(out16["losses"], outr["losses"]):
        assert abs(float(a) - float(b)) < 3e-2 * max(1.0, abs(float(b)))
    for p in m16.parameters():
        assert p.grad is None or torch.isfinite(p.grad.float()).all()
    assert m16.layers[0].wqkv.weight.grad is not None
