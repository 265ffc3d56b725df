"""CTA-pair tcgen05 GEMM (``gemm2sm``) against an fp32 matmul of the same bf16
inputs, for every operand majorness the linear layers use (forward: both
K-major; dgrad: MN-major B; wgrad: both MN-major) and every epilogue."""

import pytest
import torch

from lumenrl_b200 import ops
from lumenrl_b200.ops.ext import ext

pytestmark = pytest.mark.gpu

SHAPES = [(256, 256, 64), (512, 768, 1024), (300, 520, 4096), (1000, 1032, 136), (2048, 4096, 512),
          (64, 6144, 4096), (4096, 4096, 4096), (77, 1001, 128)]   # the last: C rows not 16-byte aligned


def _operands(M, N, K, a_mn, b_mn, dev):
    torch.manual_seed(M * 7 + N + K)
    A = torch.randn(M, K, device=dev).to(torch.bfloat16)
    B = (torch.randn(N, K, device=dev) / K ** 0.5).to(torch.bfloat16)
    a = A.t().contiguous() if a_mn else A
    b = B.t().contiguous() if b_mn else B
    return A, B, a, b


@pytest.mark.parametrize("M,N,K", SHAPES)
@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, True), (True, False)])
@pytest.mark.parametrize("bn", [128, 256, 512])
def test_gemm2sm_bf16(cuda, M, N, K, a_mn, b_mn, bn):
    if (a_mn and M % 8) or (b_mn and N % 8):
        pytest.skip("MN-major operands need a multiple of 8 along M / N")
    A, B, a, b = _operands(M, N, K, a_mn, b_mn, cuda)
    c = ext().gemm2sm(a, a_mn, b, b_mn, None, 0, bn)
    torch.cuda.synchronize()
    assert ext().gemm2sm_status() == 0
    ref = A.float() @ B.float().t()
    err = (c.float() - ref).abs().max().item()
    assert err <= 2e-2 * max(1.0, ref.abs().max().item()), err


@pytest.mark.parametrize("M,N,K", [(384, 768, 1024), (4096, 1032, 6144), (136, 256, 104)])
@pytest.mark.parametrize("bn", [0, 512])
def test_gemm2sm_fp32_and_accumulate(cuda, M, N, K, bn):
    A, B, a, b = _operands(M, N, K, True, True, cuda)
    c = torch.randn(M, N, device=cuda)
    c0 = c.clone()
    ext().gemm2sm(a, True, b, True, c, 2, bn)          # wgrad form: c += A . B^T
    f = ext().gemm2sm(A, False, B, False, None, 1, bn)  # fp32 out
    torch.cuda.synchronize()
    assert ext().gemm2sm_status() == 0
    ref = A.float() @ B.float().t()
    assert (f - ref).abs().max().item() < 2e-3 * max(1.0, ref.abs().max().item())
    assert (c - (c0 + ref)).abs().max().item() < 2e-3 * max(1.0, ref.abs().max().item())


def test_gemm2sm_strided_rows(cuda):
    """Row-strided views (a slice of a wider matrix) as both operands."""
    torch.manual_seed(3)
    big = torch.randn(512, 2048, device=cuda).to(torch.bfloat16)
    w = torch.randn(1024, 4096, device=cuda).to(torch.bfloat16)
    a, b = big[:, 512:1536], w[:, 1024:2048]
    c = ext().gemm2sm(a, False, b, False, None, 0, 0)
    torch.cuda.synchronize()
    assert ext().gemm2sm_status() == 0
    ref = a.float() @ b.float().t()
    assert (c.float() - ref).abs().max().item() <= 2e-2 * max(1.0, ref.abs().max().item())


def test_pair_gemm_from_another_thread(cuda):
    """The autograd engine runs backward GEMMs on its own thread."""
    import threading
    A, B, a, b = _operands(512, 1024, 1024, False, True, cuda)
    res = {}

    def work():
        torch.cuda.set_device(cuda)
        res["c"] = ext().gemm2sm(a, False, b, True, None, 0, 0)
        torch.cuda.synchronize()
    th = threading.Thread(target=work)
    th.start()
    th.join()
    assert ext().gemm2sm_status() == 0
    ref = A.float() @ B.float().t()
    assert (res["c"].float() - ref).abs().max().item() <= 2e-2 * max(1.0, ref.abs().max().item())


def test_linear_autograd_on_pair_gemm(cuda, monkeypatch):
    """ops.linear forward / dgrad / wgrad (main_grad accumulation) on the pair
    GEMM against fp32 autograd of the same bf16 values."""
    monkeypatch.setattr(ops, "TRAIN_GEMM", "own")
    torch.manual_seed(5)
    T, K, N = 1536, 4096, 1024
    x = torch.randn(T, K, device=cuda).to(torch.bfloat16).requires_grad_(True)
    w = (torch.randn(N, K, device=cuda) / K ** 0.5).to(torch.bfloat16).requires_grad_(True)
    w.main_grad = torch.zeros(N, K, device=cuda)
    dy = torch.randn(T, N, device=cuda).to(torch.bfloat16)
    y = ops.linear(x, w)
    y.backward(dy)
    xf, wf = x.detach().float().requires_grad_(True), w.detach().float().requires_grad_(True)
    yf = xf @ wf.t()
    yf.backward(dy.float())
    assert (y.float() - yf).abs().max().item() < 3e-2 * yf.abs().max().item()
    assert (x.grad.float() - xf.grad).abs().max().item() < 3e-2 * xf.grad.abs().max().item()
    assert (w.main_grad - wf.grad).abs().max().item() < 1e-2 * wf.grad.abs().max().item()


@pytest.mark.parametrize("T,V,H", [(300, 1000, 256), (2048, 151936, 512), (64, 4097 * 8, 128)])
def test_fused_lm_head_logprob(cuda, T, V, H):
    """Log-softmax + gather + entropy in the pair GEMM's epilogue (logits never
    written) against fp32 math on the logits the same GEMM writes as bf16 (the
    epilogue rounds each logit to bf16 exactly as that store does), and the
    logits against an fp32 matmul."""
    torch.manual_seed(T)
    h = torch.randn(T, H, device=cuda).to(torch.bfloat16)
    w = (torch.randn(V, H, device=cuda) / H ** 0.5 * 3).to(torch.bfloat16)
    tg = torch.randint(0, V, (T,), device=cuda)
    logits = ext().gemm2sm(h, False, w, False, None, 0, 256)
    ref32 = h.float() @ w.float().t()
    assert (logits.float() - ref32).abs().max().item() <= 2e-2 * ref32.abs().max().item()
    for inv_t in (1.0, 1.0 / 0.7):
        logp, ent, lse = ext().gemm2sm_logprob(h, w, tg, inv_t)
        torch.cuda.synchronize()
        assert ext().gemm2sm_status() == 0
        z = logits.float() * inv_t
        ref_lse = torch.logsumexp(z, -1)
        p = torch.softmax(z, -1)
        tol = 1e-4 * ref_lse.abs().clamp(min=1.0)       # hardware exp, other summation order
        assert bool(((lse - ref_lse).abs() <= tol).all())
        assert bool(((logp - (z.gather(1, tg[:, None]).squeeze(1) - ref_lse)).abs() <= tol).all())
        assert bool(((ent - (ref_lse - (p * z).sum(-1))).abs() <= tol).all())
