"""Persistent stream-K weight-streaming GEMM (``skinny_sk``) against an fp32
matmul of the same bf16 inputs: whole and split tiles, odd grids, repeated
calls (the workspace must be left zero) and CUDA-graph replay."""

import pytest
import torch

from lumenrl_b200.ops.ext import ext

pytestmark = pytest.mark.gpu

SHAPES = [(64, 6144, 4096), (64, 4096, 4096), (64, 24576, 4096), (64, 4096, 12288), (1, 1000, 136),
          (16, 640, 64), (33, 4096, 4096), (100, 2048, 1024), (128, 6144, 4096), (64, 151936, 4096)]


def _check(M, N, K, grid, dev, reps=2):
    torch.manual_seed(M + N + K + grid)
    x = torch.randn(M, K, device=dev).to(torch.bfloat16)
    w = (torch.randn(N, K, device=dev) / K ** 0.5).to(torch.bfloat16)
    ref = x.float() @ w.float().t()
    for _ in range(reps):
        y = ext().skinny_sk(x, w, grid)
        torch.cuda.synchronize()
        assert ext().skinny_sk_status() == 0
        err = (y.float() - ref).abs().max().item()
        assert err <= 2e-2 * max(1.0, ref.abs().max().item()), (M, N, K, grid, err)


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_skinny_sk_matches_fp32(cuda, M, N, K):
    _check(M, N, K, 0, cuda)


@pytest.mark.parametrize("grid", [1, 7, 148, 1000])
def test_skinny_sk_grids(cuda, grid):
    """Odd CTA counts put tile boundaries anywhere in a CTA's range (and more
    CTAs than work units leaves some CTAs without work)."""
    _check(64, 1536, 1024, grid, cuda, reps=3)


def test_skinny_sk_in_cuda_graph(cuda):
    torch.manual_seed(0)
    x = torch.randn(64, 4096, device=cuda).to(torch.bfloat16)
    w = (torch.randn(6144, 4096, device=cuda) / 64).to(torch.bfloat16)
    eager = ext().skinny_sk(x, w, 0)        # sizes the workspace before capture
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = ext().skinny_sk(x, w, 0)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert ext().skinny_sk_status() == 0
    # split tiles sum their partials in arrival order: equal up to fp32 rounding
    assert (out.float() - eager.float()).abs().max().item() <= 1e-2 * max(1.0, eager.float().abs().max().item())
