"""W8A8 weight-streaming decode GEMM (``skinny_fp8``): activations quantised
to 1x128 E4M3 blocks by its own quantiser launch, 128x128 E4M3 weight blocks.

Oracle: an fp32 matmul of the dequantised operands (the activation blocks
quantised by the torch reference quantiser with the same rule).  Also
checked against the two-kernel path (``quant_act_1x128`` + the block-scaled
GEMM), whole and split tiles, odd grids, repeated calls (the split-tile
workspace must be left zero) and CUDA-graph replay."""

import pytest
import torch

from lumenrl_b200.ops.ext import ext
from lumenrl_b200.quant.fp8 import (dequant_128x128, dequant_1x128, quant_1x128_ref, quant_act_1x128,
                                    quant_weight_128x128)

pytestmark = pytest.mark.gpu

# (M, N, K): the Qwen3-8B decode linears at 64 rows, a 32-row bucket, N not
# a multiple of 128, one K block
SHAPES = [(64, 6144, 4096), (64, 4096, 4096), (64, 24576, 4096), (64, 4096, 12288), (33, 4096, 4096),
          (1, 1000, 256), (17, 640, 128), (64, 2048, 1024)]


def _operands(M, N, K, dev, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = (torch.randn(M, K, generator=g) * torch.rand(M, 1, generator=g) * 4).to(torch.bfloat16).to(dev)
    x[0, :128] = 0                      # an all-zero activation block (scale 1, zeros out)
    w = (torch.randn(N, K, generator=g) / K ** 0.5).to(torch.bfloat16).to(dev)
    qw, sw = quant_weight_128x128(w)
    return x, qw, sw


def _oracle(x, qw, sw):
    qx, sx = quant_1x128_ref(x.float().cpu().to(torch.bfloat16))
    return (dequant_1x128(qx, sx) @ dequant_128x128(qw.cpu(), sw.cpu()).t()).to(x.device)


def _check(M, N, K, grid, dev, reps=2, seed=0):
    x, qw, sw = _operands(M, N, K, dev, seed + M + N + K)
    ref = _oracle(x, qw, sw)
    qx, sx = quant_act_1x128(x)
    two_kernel = ext().fp8_gemm(qx, sx, qw, sw, torch.zeros(1, dtype=torch.int32, device=dev)).float()
    tol = 1e-2 * max(1.0, ref.abs().max().item())
    for _ in range(reps):
        y = ext().skinny_fp8(x, qw, sw, grid)
        torch.cuda.synchronize()
        assert ext().skinny_fp8_status() == 0
        assert y.shape == (M, N) and y.dtype == torch.bfloat16
        err = (y.float() - ref).abs().max().item()
        assert err <= tol, (M, N, K, grid, err)
        assert (y.float() - two_kernel).abs().max().item() <= tol


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_skinny_fp8_matches_dequantised_fp32(cuda, M, N, K):
    _check(M, N, K, 0, cuda)


@pytest.mark.parametrize("grid", [1, 7, 148, 5000])
def test_skinny_fp8_grids(cuda, grid):
    """Odd CTA counts put tile boundaries anywhere in a CTA's range; more CTAs
    than work units are clamped to one unit per CTA."""
    _check(64, 1536, 1024, grid, cuda, reps=3)


def test_skinny_fp8_in_cuda_graph(cuda):
    x, qw, sw = _operands(64, 6144, 4096, cuda, 5)
    eager = ext().skinny_fp8(x, qw, sw, 0)      # sizes the workspace before capture
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = ext().skinny_fp8(x, qw, sw, 0)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert ext().skinny_fp8_status() == 0
    assert (out.float() - eager.float()).abs().max().item() <= 1e-2 * max(1.0, eager.float().abs().max().item())


def test_fp8_rollout_decode_linear_uses_stream_kernel(cuda):
    """The FP8 rollout quantiser's decode linears go through the stream kernel
    and agree with its prefill path (two-kernel GEMM) on the same rows."""
    from lumenrl_b200.quant.fp8 import FP8Config, FP8RolloutQuantizer
    q = FP8RolloutQuantizer(FP8Config(), num_layers=1)
    x, qw, sw = _operands(64, 4096, 4096, cuda, 9)
    q.weights["layers.0.w2"] = (qw, sw)
    dec = q.linear("layers.0.w2", x, None, decode=True)
    pre = q.linear("layers.0.w2", x, None, decode=False)
    tol = 1e-2 * max(1.0, pre.float().abs().max().item())
    assert (dec.float() - pre.float()).abs().max().item() <= tol
