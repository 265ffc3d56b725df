"""Bounds-checked NVLink kernels (``lumenrl_b200._C_bounds``, built with
-DLRL_DEBUG_BOUNDS) on one GPU.

Each case hands a kernel an extent that is smaller than what its arguments
claim: the registered range is a prefix of a larger allocation, so the checked
kernel must skip the accesses past the prefix and record the site code, while
the rest of the allocation (the guard) stays untouched.  Every access the
arguments describe lies inside the allocation, so the cases stay safe even if
a check were missing; the guard contents are what detect one."""

import importlib

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def B(cuda):
    mod = importlib.import_module("lumenrl_b200._C_bounds")
    assert mod.debug_bounds_build()
    return mod


def _fresh(B):
    torch.cuda.synchronize()
    B.bounds_reset()
    torch.cuda.synchronize()


def test_p2p_push_past_the_destination(B, cuda):
    big = torch.zeros(4096 + 1024, dtype=torch.float32, device=cuda)
    flag = torch.zeros(4, dtype=torch.int32, device=cuda)
    counter = torch.zeros(1, dtype=torch.int32, device=cuda)
    B.bounds_register(big.data_ptr(), 4096 * 4)
    B.bounds_register(flag.data_ptr(), 16)
    try:
        _fresh(B)
        B.p2p_push(torch.ones(4096 + 512, device=cuda), big.data_ptr(), flag.data_ptr(), 1, counter)
        torch.cuda.synchronize()
        assert B.bounds_status() == 905
        assert float(big.abs().sum()) == 0.0          # nothing stored: the range does not fit
        assert int(flag[0]) == 1                      # the flag store itself was in bounds
        _fresh(B)
        B.p2p_push(torch.ones(4096, device=cuda), big.data_ptr(), flag.data_ptr(), 2, counter)
        torch.cuda.synchronize()
        assert B.bounds_status() == 0
        assert bool((big[:4096] == 1).all()) and float(big[4096:].abs().sum()) == 0.0
        assert int(flag[0]) == 2
    finally:
        B.bounds_unregister(big.data_ptr())
        B.bounds_unregister(flag.data_ptr())


def test_ep_scatter_rows_past_capacity_and_bad_source_row(B, cuda):
    H, cap = 64, 8
    buf = torch.zeros(2 * cap, H, dtype=torch.bfloat16, device=cuda)
    sig = torch.zeros(int(B.ep_flag_slots()), dtype=torch.int32, device=cuda)
    B.bounds_register(buf.data_ptr(), cap * H * 2)
    B.bounds_register(sig.data_ptr(), sig.numel() * 4)
    src_all = torch.randn(8, H, device=cuda).to(torch.bfloat16)
    src = src_all[:4]
    counter = torch.zeros(1, dtype=torch.int32, device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    rank0 = torch.zeros(4, dtype=torch.int32, device=cuda)
    try:
        # the claimed capacity (2 * cap) exceeds the registered one (cap)
        _fresh(B)
        rows = torch.tensor([0, 3, 9, 12], dtype=torch.int32, device=cuda)
        B.ep_scatter_rows(src, None, rank0, rows, [buf.data_ptr()], 2 * cap, [sig.data_ptr()], 0, 0, 1, counter,
                          status)
        torch.cuda.synchronize()
        assert B.bounds_status() == 903 and int(status[0]) == 0
        assert torch.equal(buf[0], src[0]) and torch.equal(buf[3], src[1])
        assert float(buf[cap:].float().abs().sum()) == 0.0
        assert int(sig[0]) == 1                       # flag published in bounds
        # a source row past the source tensor (still inside src_all)
        buf.zero_()
        _fresh(B)
        B.ep_scatter_rows(src, torch.tensor([0, 7], dtype=torch.int64, device=cuda), rank0[:2],
                          torch.tensor([1, 2], dtype=torch.int32, device=cuda), [buf.data_ptr()], cap,
                          [sig.data_ptr()], 0, 0, 2, counter, status)
        torch.cuda.synchronize()
        assert B.bounds_status() == 904
        assert torch.equal(buf[1], src[0]) and float(buf[2].float().abs().sum()) == 0.0
    finally:
        B.bounds_unregister(buf.data_ptr())
        B.bounds_unregister(sig.data_ptr())


def test_allreduce_and_rs_norm_past_the_buffer(B, cuda):
    words = int(B.symm_signal_words())
    sig = torch.zeros(words, dtype=torch.int32, device=cuda)
    B.bounds_register(sig.data_ptr(), words * 4)
    buf = torch.ones(2048 + 1024, dtype=torch.float32, device=cuda)
    B.bounds_register(buf.data_ptr(), 2048 * 4)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    wait = int(0.5 * 2.0e9)
    try:
        # one rank, n past the registered 2048 elements
        _fresh(B)
        B.nvlink_allreduce([buf.data_ptr()], [sig.data_ptr()], 0, 2048 + 512, 2.0, 1, status, wait)
        torch.cuda.synchronize()
        assert int(status[0]) == 0 and B.bounds_status() == 909
        assert bool((buf[:2048] == 2).all()) and bool((buf[2048:] == 1).all())
        # rs_norm: shard [512, 1536) of a buffer registered as 1024 elements
        grads = torch.arange(2048, dtype=torch.float32, device=cuda)
        B.bounds_register(grads.data_ptr(), 1024 * 4)
        out = torch.full((1024,), -1.0, device=cuda)
        _fresh(B)
        B.rs_norm([grads.data_ptr()], [sig.data_ptr()], 0, 512, 1024, out, 1, status, wait)
        torch.cuda.synchronize()
        B.bounds_unregister(grads.data_ptr())
        assert int(status[0]) == 0 and B.bounds_status() == 907
        assert torch.equal(out[:512], grads[512:1024]) and float(out[512:].abs().sum()) == 0.0
        # in bounds: no violation, same result as the ordinary build's contract
        buf.fill_(3.0)
        _fresh(B)
        B.nvlink_allreduce([buf.data_ptr()], [sig.data_ptr()], 0, 2048, 0.5, 2, status, wait)
        torch.cuda.synchronize()
        assert int(status[0]) == 0 and B.bounds_status() == 0
        assert bool((buf[:2048] == 1.5).all()) and bool((buf[2048:] == 3).all())
    finally:
        B.bounds_unregister(buf.data_ptr())
        B.bounds_unregister(sig.data_ptr())


def test_ext_routes_comm_ops_to_the_bounds_module(cuda, monkeypatch):
    ext_mod = importlib.import_module("lumenrl_b200.ops.ext")
    saved = (ext_mod._MOD, ext_mod._ERR)
    try:
        monkeypatch.setenv("LRL_DEBUG_BOUNDS", "1")
        ext_mod._MOD, ext_mod._ERR = None, None
        e = ext_mod.ext()
        assert e.debug_bounds_build() is True
        ext_mod.bounds_clear()
        assert ext_mod.bounds_error() == 0
        assert callable(e.rmsnorm_fwd)               # everything else still comes from _C
    finally:
        ext_mod._MOD, ext_mod._ERR = saved
