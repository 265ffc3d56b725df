"""Hand-written tcgen05 GEMM against an fp32 matmul of the same bf16 inputs."""

import pytest
import torch

from lumenrl_b200 import ops
from lumenrl_b200.ops.ext import ext

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,N,K,bn", [(128, 128, 64, 128), (256, 512, 256, 128), (300, 640, 4096, 0),
                                      (64, 6144, 4096, 0), (1024, 2048, 512, 256), (77, 1000 * 8, 136, 128),
                                      (4096, 4096, 4096, 0)])
def test_tc_gemm_bf16(cuda, M, N, K, bn):
    torch.manual_seed(0)
    a = torch.randn(M, K, device=cuda).to(torch.bfloat16)
    b = (torch.randn(N, K, device=cuda) / K ** 0.5).to(torch.bfloat16)
    c = ops.tc_gemm(a, b, bn=bn)
    torch.cuda.synchronize()
    assert ops.tc_gemm_status() == 0
    ref = a.float() @ b.float().t()
    err = (c.float() - ref).abs().max().item()
    assert err <= 2e-2 * max(1.0, ref.abs().max().item()), err


def test_tc_gemm_fp32_accumulate(cuda):
    torch.manual_seed(1)
    M, N, K = 384, 768, 1024
    a = torch.randn(M, K, device=cuda).to(torch.bfloat16)
    b = torch.randn(N, K, device=cuda).to(torch.bfloat16)
    c = torch.randn(M, N, device=cuda)
    c0 = c.clone()
    ops.tc_gemm(a, b, out=c, accumulate=True)
    f = ops.tc_gemm(a, b, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert ops.tc_gemm_status() == 0
    ref = a.float() @ b.float().t()
    assert (f - ref).abs().max().item() < 1e-2
    assert (c - (c0 + ref)).abs().max().item() < 1e-2


@pytest.mark.parametrize("M,N,K", [(64, 6144, 4096), (3, 1000 * 8, 520), (128, 512, 4096)])
def test_tc_gemm_splitk(cuda, M, N, K):
    from lumenrl_b200.ops.ext import ext
    torch.manual_seed(0)
    a = torch.randn(M, K, device=cuda).to(torch.bfloat16)
    b = (torch.randn(N, K, device=cuda) / K ** 0.5).to(torch.bfloat16)
    for splits in (0, 3, 100):
        c = ext().tc_gemm_splitk(a, b, splits)
        torch.cuda.synchronize()
        assert ops.tc_gemm_status() == 0
        ref = a.float() @ b.float().t()
        assert (c - ref).abs().max().item() <= 1e-2 * max(1.0, ref.abs().max().item())


@pytest.mark.parametrize("M", [1, 16, 33, 64, 100, 128, 200, 256])
@pytest.mark.parametrize("N,K", [(6144, 4096), (1000, 72), (4096, 12288)])
def test_skinny_gemm_decode_sizes(cuda, M, N, K):
    """Weight-streaming GEMM (operands swapped, K split over a cluster with a
    distributed-shared-memory reduction) against an fp32 reference."""
    torch.manual_seed(M + N)
    x = torch.randn(M, K, device=cuda).to(torch.bfloat16)
    w = (torch.randn(N, K, device=cuda) / K ** 0.5).to(torch.bfloat16)
    ref = x.float() @ w.float().t()
    for ks in (0, 1, 2, 3, 8):
        y = ops.skinny_linear(x, w, ks)
        torch.cuda.synchronize()
        assert ext().skinny_gemm_status() == 0
        assert y.shape == (M, N)
        assert torch.allclose(y.float(), ref, atol=2e-2, rtol=2e-2), (ks, (y.float() - ref).abs().max())
