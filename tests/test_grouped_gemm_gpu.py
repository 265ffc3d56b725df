"""tcgen05 grouped expert GEMM against per-expert fp32 GEMMs: ragged and
empty experts, rows past the last expert, forward, input and weight
gradients; and the MoE block through it against the per-expert loop."""

import pytest
import torch

from lumenrl_b200.models.moe import grouped_linear, grouped_linear_device

pytestmark = pytest.mark.gpu


def _offsets(counts, dev):
    o = torch.zeros(len(counts) + 1, dtype=torch.int32, device=dev)
    o[1:] = torch.cumsum(torch.tensor(counts, device=dev), 0)
    return o


@pytest.mark.parametrize("E,N,K,counts", [(4, 256, 512, [130, 0, 1, 300]), (8, 128, 256, [17] * 8),
                                          (16, 384, 2048, [0, 0, 500, 3, 0, 129, 128, 127, 1, 2, 3, 4, 5, 6, 7, 8])])
def test_grouped_gemm_matches_per_expert(cuda, E, N, K, counts):
    torch.manual_seed(0)
    T = sum(counts) + 37   # trailing rows belong to no expert
    x = torch.randn(T, K, device=cuda).to(torch.bfloat16)
    w = (torch.randn(E, N, K, device=cuda) / K ** 0.5).to(torch.bfloat16)
    offs = _offsets(counts, cuda)
    xr = x.clone().requires_grad_(True)
    wr = torch.nn.Parameter(w.clone())
    y = grouped_linear_device(xr, wr, offs)
    dy = torch.randn_like(y)
    y.backward(dy)
    torch.cuda.synchronize()
    from lumenrl_b200.ops.ext import ext
    assert ext().grouped_gemm_status() == 0
    off = offs.tolist()
    n = off[-1]
    for e in range(E):
        a, b = off[e], off[e + 1]
        if b > a:
            ref = x[a:b].float() @ w[e].float().t()
            assert torch.allclose(y[a:b].float(), ref, atol=3e-2, rtol=2e-2), e
            gx = dy[a:b].float() @ w[e].float()
            assert torch.allclose(xr.grad[a:b].float(), gx, atol=5e-2, rtol=3e-2), e
            gw = dy[a:b].float().t() @ x[a:b].float()
            assert torch.allclose(wr.grad[e].float(), gw, atol=0.3, rtol=3e-2), e
        else:
            assert wr.grad[e].abs().max() == 0
    assert n <= T


def test_moe_block_tc_matches_loop(cuda):
    from lumenrl_b200.models.config import tiny_qwen3_moe
    from lumenrl_b200.models.moe import moe_forward
    from lumenrl_b200.models.qwen3 import Qwen3Model
    import lumenrl_b200.models.moe as moe
    m = Qwen3Model(tiny_qwen3_moe(), device=cuda, dtype=torch.bfloat16, requires_grad=False)
    m.init_weights(0)
    h = torch.randn(300, m.args.hidden_size, device=cuda).to(torch.bfloat16)
    out_tc, _ = moe_forward(m, 0, h)
    orig = moe._use_tc_grouped
    moe._use_tc_grouped = lambda *a: False
    try:
        out_loop, _ = moe_forward(m, 0, h)
    finally:
        moe._use_tc_grouped = orig
    assert torch.allclose(out_tc.float(), out_loop.float(), atol=2e-2, rtol=2e-2)
