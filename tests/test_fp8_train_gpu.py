"""Hybrid FP8 training kernels against fp32 references on the same quantised
values: the block-scaled tcgen05 GEMM in every operand-format combination
(E4M3 / E5M2), with 128x128 or per-row B scales and the fp32 accumulate
epilogue; the transposed 1x128 quantiser; and the FP8 linear's forward,
dgrad and wgrad against fp32 autograd."""

import pytest
import torch

from lumenrl_b200.quant.fp8 import (E4M3, E5M2, FP8Config, FP8TrainingManager, dequant_1x128, dequant_128x128,
                                    fp8_gemm_status, fp8_matmul, quant_1x128_ref, quant_act_1x128, quant_t_1x128,
                                    quant_weight_128x128)

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("fa,fb", [(E4M3, E4M3), (E5M2, E4M3), (E4M3, E5M2), (E5M2, E5M2)])
@pytest.mark.parametrize("M,N,K", [(256, 384, 512), (300, 1000, 4096), (77, 136, 144)])
def test_fp8_block_scaled_gemm_formats(cuda, fa, fb, M, N, K):
    torch.manual_seed(M + N)
    a = (torch.randn(M, K, device=cuda) * 3).to(torch.bfloat16)
    b = (torch.randn(N, K, device=cuda) / 8).to(torch.bfloat16)
    qa, sa = quant_act_1x128(a, fa)
    qb, sb = quant_weight_128x128(b, fb)
    ref = dequant_1x128(qa, sa) @ dequant_128x128(qb, sb).t()
    out = fp8_matmul(qa, sa, qb, sb)
    torch.cuda.synchronize()
    assert fp8_gemm_status() == 0
    assert (out.float() - ref).abs().max().item() <= 1e-2 * ref.abs().max().item() + 1e-3


@pytest.mark.parametrize("R,C", [(1536, 4096), (200, 136), (7, 64)])
def test_transposed_quantiser_matches_reference(cuda, R, C):
    """Scales equal the reference up to the last bit (division vs multiply
    by the reciprocal) and every dequantised value is within half an FP8
    step of the input."""
    torch.manual_seed(R)
    x = torch.randn(R, C, device=cuda).to(torch.bfloat16)
    Rpad = (R + 127) // 128 * 128
    xt = torch.nn.functional.pad(x.float().t(), (0, Rpad - R))
    for dt, half_step in ((E4M3, 2.0 ** -4), (E5M2, 2.0 ** -3)):
        q, s = quant_t_1x128(x, dt)
        qr, sr = quant_1x128_ref(xt, dt)
        assert q.shape == (C, Rpad) and s.shape == (C, Rpad // 128)
        assert torch.allclose(s, sr.to(s.device), rtol=1e-6, atol=0)
        deq = dequant_1x128(q, s)
        tiny = s.repeat_interleave(128, -1) * 2.0 ** -9       # subnormal spacing
        assert bool(((deq - xt).abs() <= half_step * xt.abs() + tiny).all())
        assert (q.view(torch.uint8) != qr.to(q.device).view(torch.uint8)).float().mean().item() < 1e-2
        qk, sk = quant_t_1x128(x, dt, kb_major=True)
        assert sk.shape == (Rpad // 128, (C + 127) // 128 * 128)
        assert torch.equal(sk[:, :C].t().contiguous(), s)


def test_row_scaled_wgrad_gemm_accumulates(cuda):
    """dW += dY^T X with both operands quantised along tokens (E5M2 x E4M3)."""
    torch.manual_seed(0)
    T, N, K = 1000, 384, 264
    dy = (torch.randn(T, N, device=cuda) / 10).to(torch.bfloat16)
    x = torch.randn(T, K, device=cuda).to(torch.bfloat16)
    qdt, sdt = quant_t_1x128(dy, E5M2)
    qxt, sxt = quant_t_1x128(x, E4M3, kb_major=True)
    acc = torch.randn(N, K, device=cuda)
    acc0 = acc.clone()
    fp8_matmul(qdt, sdt, qxt, sxt, out=acc, b_row=True)
    torch.cuda.synchronize()
    assert fp8_gemm_status() == 0
    ref = dequant_1x128(qdt, sdt) @ dequant_1x128(qxt, sxt[:, :K].t()).t()
    assert (acc - acc0 - ref).abs().max().item() <= 1e-2 * ref.abs().max().item()


def test_fp8_linear_forward_dgrad_wgrad(cuda):
    torch.manual_seed(1)
    T, K, N = 1536, 1024, 768
    mgr = FP8TrainingManager(FP8Config(precision="hybrid"))
    x = torch.randn(T, K, device=cuda).to(torch.bfloat16).requires_grad_(True)
    w = (torch.randn(N, K, device=cuda) / K ** 0.5).to(torch.bfloat16).requires_grad_(True)
    w.main_grad = torch.zeros(N, K, device=cuda)
    dy = torch.randn(T, N, device=cuda).to(torch.bfloat16)
    y = mgr.linear("layers.0.wqkv", x, w)
    y.backward(dy)
    torch.cuda.synchronize()
    assert fp8_gemm_status() == 0
    xf, wf = x.detach().float().requires_grad_(True), w.detach().float().requires_grad_(True)
    (xf @ wf.t()).backward(dy.float())
    yf = xf.detach() @ wf.detach().t()
    rel = lambda a, b: ((a.float() - b).norm() / b.norm()).item()   # noqa: E731
    assert rel(y, yf) < 0.05           # E4M3 operands: a few % relative error
    assert rel(x.grad, xf.grad) < 0.08  # E5M2 gradient
    assert rel(w.main_grad, wf.grad) < 0.08
