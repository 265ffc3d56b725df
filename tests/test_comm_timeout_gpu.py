"""Failure detection without a GPU fault: a cross-rank flag that nothing sets.

Two "ranks" are emulated on ONE GPU: rank 1's signal area is a local buffer
that no kernel ever writes, so rank 0's barrier must give up after its short
bound, record the barrier slot in the status word and return; the context
stays usable for the next kernel."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_barrier_wait_expires_with_status(cuda):
    from lumenrl_b200.ops.ext import ext
    e = ext()
    n = 4096
    g0, g1 = e.symm_malloc(n * 4)[0], e.symm_malloc(n * 4)[0]
    w = int(e.symm_signal_words())
    s0, s1 = e.symm_malloc(w * 4)[0], e.symm_malloc(w * 4)[0]
    out = torch.zeros(n // 2, device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    try:
        e.rs_norm([g0, g1], [s0, s1], 0, 0, n // 2, out, 1, status, int(0.2 * 2.0e9))
        torch.cuda.synchronize()
        assert int(status.item()) == 100          # slot-0 barrier expired
        x = torch.ones(1000, device=cuda)
        assert float(x.sum()) == 1000.0            # the context is still healthy
    finally:
        for p in (g0, g1, s0, s1):
            e.symm_free(p)
