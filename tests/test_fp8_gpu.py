"""FP8 blockwise quantisers and the tcgen05 kind::f8f6f4 block-scaled GEMM."""

import pytest
import torch

from lumenrl_b200 import ops
from lumenrl_b200.quant import fp8 as F

pytestmark = pytest.mark.gpu


def test_quantizers_match_reference(cuda):
    torch.manual_seed(0)
    x = torch.randn(37, 1000, device=cuda).to(torch.bfloat16)
    q, s = F.quant_act_1x128(x)
    qr, sr = F.quant_1x128_ref(x.cpu())
    assert torch.allclose(s.cpu(), sr, rtol=1e-6)
    assert (q.float().cpu() - qr.float()).abs().max().item() <= 32.0     # one e4m3 ulp near 448
    w = torch.randn(300, 384, device=cuda).to(torch.bfloat16)
    qw, sw = F.quant_weight_128x128(w)
    qwr, swr = F.quant_128x128_ref(w.cpu())
    assert torch.allclose(sw.cpu(), swr, rtol=1e-6)
    err = (F.dequant_128x128(qw.cpu(), sw.cpu()) - w.float().cpu()).abs().max().item()
    assert err <= 0.07 * w.float().abs().max().item()


@pytest.mark.parametrize("M,N,K", [(128, 128, 128), (200, 384, 512), (64, 6144, 4096), (1024, 2048, 1024)])
def test_fp8_gemm_blockwise(cuda, M, N, K):
    torch.manual_seed(0)
    x = torch.randn(M, K, device=cuda).to(torch.bfloat16)
    w = (torch.randn(N, K, device=cuda) / K ** 0.5).to(torch.bfloat16)
    qx, sx = F.quant_act_1x128(x)
    qw, sw = F.quant_weight_128x128(w)
    out = ops.fp8_gemm_blockwise(x, qw, sw, qx, sx)
    torch.cuda.synchronize()
    assert ops.fp8_gemm_status() == 0
    ref = F.dequant_1x128(qx, sx) @ F.dequant_128x128(qw, sw).t()
    err = (out.float() - ref).abs().max().item()
    assert err <= 2e-2 * max(1.0, ref.abs().max().item()), err
