"""Loader for the in-tree CUDA extension ``lumenrl_b200._C``.

The extension is built in place (``python setup.py build_ext --inplace`` or
``__graft_entry__.build()``) so the ``.so`` sits next to the package and is
what every process on a GPU machine imports.  There is no fallback: a CUDA
tensor reaching an op without the extension raises ``RuntimeError``.
"""

from __future__ import annotations

import importlib
import os

_MOD = None
_ERR: Exception | None = None
LAUNCHES = [0]   # kernels of this extension launched (graph replays add their captured count)


# host-only entry points (no kernel) and ops that launch two kernels
_NO_KERNEL = {"symm_malloc", "symm_open", "symm_close", "symm_free", "symm_tensor", "symm_signal_words",
              "bounds_register", "bounds_unregister", "bounds_lookup", "bounds_status", "bounds_reset",
              "debug_bounds_build",
              "ep_flag_slots", "tc_gemm_status", "skinny_gemm_status", "skinny_sk_status", "grouped_gemm_status", "decode_tma_status",
              "fa_fwd_status", "fa_bwd_status", "gemm2sm_status", "install_segv_backtrace"}
_TWO_KERNELS = {"fa_fwd", "paged_decode_attn_shared", "paged_decode_attn_tma", "paged_decode_attn_shared_tma", "gemm_rs"}


def _kernels(name: str, a: tuple) -> int:
    if name in _NO_KERNEL:
        return 0
    if name in _TWO_KERNELS:
        return 2
    if name == "fa_bwd":                # three transposes, the lse/D pass, the dQ and the dK/dV kernels
        return 6
    if name == "paged_decode_attn":     # + the split combine, unless one split covers the context
        return 2
    if name == "sample":                # split-row sampler (top_p = 1, bf16, large vocab) is two kernels
        logits, top_p = a[0], a[2]
        return 2 if (top_p >= 1.0 and str(logits.dtype) == "torch.bfloat16" and logits.shape[-1] >= 16384) else 1
    return 1


class _Counted:
    """Proxy that counts the kernels the extension launches (an estimate for
    the split decode attention, whose combine pass is skipped when a single
    split covers the context).  With a bounds module (``LRL_DEBUG_BOUNDS=1``)
    every op that module defines -- the NVLink comm kernels, the symmetric
    buffer plumbing and the bounds registry -- resolves there."""

    def __init__(self, mod, bounds=None) -> None:
        self._mod = mod
        self._bounds = bounds

    def __getattr__(self, name):
        src = self._bounds if self._bounds is not None and hasattr(self._bounds, name) else self._mod
        fn = getattr(src, name)
        if not callable(fn):
            return fn

        def call(*a, **k):
            LAUNCHES[0] += _kernels(name, a)
            return fn(*a, **k)
        return call


def _load():
    global _MOD, _ERR
    if _MOD is not None or _ERR is not None:
        return
    try:
        import torch  # noqa: F401  (loads libc10/libtorch for the extension)
        mod = importlib.import_module("lumenrl_b200._C")
    except Exception as e:  # pragma: no cover - depends on the build
        _ERR = e
        return
    bounds = None
    if debug_bounds_requested():
        # no fallback: a run that asked for checked kernels must get them
        bounds = importlib.import_module("lumenrl_b200._C_bounds")
        import torch
        if torch.cuda.is_available():
            # allocates this device's bounds status word now, outside any
            # CUDA-graph capture (the checked kernels write it)
            bounds.bounds_reset()
    _MOD = _Counted(mod, bounds)


def debug_bounds_requested() -> bool:
    """``LRL_DEBUG_BOUNDS=1``: the NVLink comm kernels come from
    ``lumenrl_b200._C_bounds``, where every peer and signal-area access is
    checked against its buffer's registered extent; a violation is skipped and
    recorded (``bounds_error()``) instead of faulting a GPU."""
    return os.environ.get("LRL_DEBUG_BOUNDS", "0") == "1"


def bounds_error() -> int:
    """Site code of the first out-of-bounds access the checked comm kernels
    recorded on the current device since the last ``bounds_clear()`` (0 =
    none, always 0 without ``LRL_DEBUG_BOUNDS=1``).  Synchronises."""
    return int(ext().bounds_status())


def bounds_clear() -> None:
    ext().bounds_reset()


def has_ext() -> bool:
    _load()
    return _MOD is not None


def ext():
    _load()
    if _MOD is None:
        raise RuntimeError(
            "lumenrl_b200._C (the sm_100a kernels) is not built or failed to load: "
            f"{_ERR!r}. Build it with `python setup.py build_ext --inplace`.")
    return _MOD
