"""The scratch-free decode-attention entry point, called through its exported
C symbol, against the allocating entry point.

Some callers of this library cannot allocate GPU memory while they run (a
program that fixes its device memory at start-up, or a plugin that must not
use its host runtime's allocator).  ``lrl_paged_decode_attn_noalloc`` serves
them: it takes its split-K scratch from a static device array instead of an
allocator.  This file is named so that pytest collects it last.
"""

import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    import lumenrl_b200._C as C
    lib = ctypes.CDLL(C.__file__)
    f = lib.lrl_paged_decode_attn_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_int] * 6 + [ctypes.c_float] * 3 + [ctypes.c_int, ctypes.c_void_p]
    lib.lrl_decode_noalloc_last_error.restype = ctypes.c_char_p
    lib.lrl_decode_noalloc_scratch_bytes.restype = ctypes.c_size_t
    return lib


def _case(dev, kv_dtype, B, Hq, Hk, bs, maxlen, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    D = 128
    lens = torch.randint(1, maxlen + 1, (B,), generator=g).to(torch.int32)
    lens[0] = maxlen
    mb = (maxlen + bs - 1) // bs
    nblocks = B * mb + 2
    bt = (torch.randperm(nblocks - 1, generator=g)[: B * mb] + 1).view(B, mb).to(torch.int32)
    kc = torch.randn(nblocks, bs, Hk, D, generator=g).to(kv_dtype)
    vc = torch.randn(nblocks, bs, Hk, D, generator=g).to(kv_dtype)
    q = torch.randn(B, Hq, D, generator=g).to(torch.bfloat16)
    return [t.to(dev) for t in (q, kc, vc, bt, lens)]


@pytest.mark.parametrize("kv_dtype", [torch.bfloat16, torch.float8_e4m3fn])
def test_noalloc_entry_matches_allocating_entry(cuda, kv_dtype):
    from lumenrl_b200.ops.ext import ext
    lib = _lib()
    assert lib.lrl_decode_noalloc_scratch_bytes() == 8 * 1024 * 1024
    B, Hq, Hk, bs, maxlen = 3, 32, 8, 64, 700      # few (seq, head) pairs -> split-K uses the scratch
    ks, vs = (0.5, 2.0) if kv_dtype != torch.bfloat16 else (1.0, 1.0)
    scale = 1.0 / math.sqrt(128)
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):                         # two calls in a row share the static scratch
        q, kc, vc, bt, lens = _case(cuda, kv_dtype, B, Hq, Hk, bs, maxlen, seed=call)
        want = ext().paged_decode_attn(q, kc, vc, bt, lens, scale, ks, vs, maxlen)
        out = torch.empty_like(q)
        rc = lib.lrl_paged_decode_attn_noalloc(
            q.data_ptr(), kc.data_ptr(), vc.data_ptr(), bt.data_ptr(), lens.data_ptr(), out.data_ptr(),
            B, Hq, Hk, bs, bt.shape[1], int(kv_dtype != torch.bfloat16), scale, ks, vs, maxlen, stream)
        assert rc == 0, lib.lrl_decode_noalloc_last_error()
        torch.cuda.synchronize()
        err = (out.float() - want.float()).abs().max().item()
        assert err <= 2e-2, f"call {call}: max abs err {err}"


def test_noalloc_single_split_shape(cuda):
    """A context of one 64-token tile needs no split (no scratch is touched);
    the result still matches the allocating entry point, twice in a row."""
    from lumenrl_b200.ops.ext import ext
    lib = _lib()
    B, Hq, Hk, bs, maxlen = 4, 32, 8, 16, 60
    scale = 1.0 / math.sqrt(128)
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        q, kc, vc, bt, lens = _case(cuda, torch.bfloat16, B, Hq, Hk, bs, maxlen, seed=10 + call)
        want = ext().paged_decode_attn(q, kc, vc, bt, lens, scale, 1.0, 1.0, maxlen)
        out = torch.empty_like(q)
        rc = lib.lrl_paged_decode_attn_noalloc(
            q.data_ptr(), kc.data_ptr(), vc.data_ptr(), bt.data_ptr(), lens.data_ptr(), out.data_ptr(),
            B, Hq, Hk, bs, bt.shape[1], 0, scale, 1.0, 1.0, maxlen, stream)
        assert rc == 0, lib.lrl_decode_noalloc_last_error()
        torch.cuda.synchronize()
        assert (out.float() - want.float()).abs().max().item() <= 2e-2


def _scratch_need_bytes(B, Hq, Hk, maxlen, sms):
    """Split-K scratch the entry point needs for a shape (its split rule:
    about four CTAs per SM, at most 32 splits and one per 64-token tile)."""
    tiles = -(-maxlen // 64)
    ctas = B * Hk
    nsplit = max(1, min(32, tiles, -(-4 * sms // ctas)))
    return 0 if nsplit == 1 else nsplit * B * Hq * 129 * 4


def test_noalloc_rejects_oversize_and_null_without_launching(cuda):
    """Shapes needing more split-K scratch than the static array, and null
    pointers, return cudaErrorInvalidValue (1) with a message and launch
    nothing: the output keeps its sentinel."""
    lib = _lib()
    sms = torch.cuda.get_device_properties(cuda).multi_processor_count
    cap = lib.lrl_decode_noalloc_scratch_bytes()
    Hq, Hk, bs, maxlen = 128, 8, 64, 256
    B = next(b for b in range(1, 4096) if _scratch_need_bytes(b, Hq, Hk, maxlen, sms) > cap)
    q, kc, vc, bt, lens = _case(cuda, torch.bfloat16, B, Hq, Hk, bs, maxlen, seed=3)
    out = torch.full_like(q, 7.0)
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.lrl_paged_decode_attn_noalloc(
        q.data_ptr(), kc.data_ptr(), vc.data_ptr(), bt.data_ptr(), lens.data_ptr(), out.data_ptr(),
        B, Hq, Hk, bs, bt.shape[1], 0, 1.0 / math.sqrt(128), 1.0, 1.0, maxlen, stream)
    assert rc == 1
    assert b"exceeds" in lib.lrl_decode_noalloc_last_error()
    rc = lib.lrl_paged_decode_attn_noalloc(
        None, kc.data_ptr(), vc.data_ptr(), bt.data_ptr(), lens.data_ptr(), out.data_ptr(),
        B, Hq, Hk, bs, bt.shape[1], 0, 1.0 / math.sqrt(128), 1.0, 1.0, maxlen, stream)
    assert rc == 1
    assert b"null" in lib.lrl_decode_noalloc_last_error()
    torch.cuda.synchronize()
    assert bool((out.float() == 7.0).all())
