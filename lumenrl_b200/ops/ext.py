"""Loader for the in-tree CUDA extension ``lumenrl_b200._C``.

The extension is built in place (``python setup.py build_ext --inplace`` or
``__graft_entry__.build()``) so the ``.so`` sits next to the package and is
what every process on a GPU machine imports.  There is no fallback: a CUDA
tensor reaching an op without the extension raises ``RuntimeError``.
"""

from __future__ import annotations

import importlib

_MOD = None
_ERR: Exception | None = None
LAUNCHES = [0]   # kernels of this extension launched (graph replays add their captured count)


class _Counted:
    """Proxy that counts launches of the extension's kernels.  Each op call is
    one kernel launch except the split decode attention (two)."""

    def __init__(self, mod) -> None:
        self._mod = mod

    def __getattr__(self, name):
        fn = getattr(self._mod, name)
        if not callable(fn):
            return fn

        def call(*a, **k):
            LAUNCHES[0] += 1
            return fn(*a, **k)
        return call


def _load():
    global _MOD, _ERR
    if _MOD is not None or _ERR is not None:
        return
    try:
        import torch  # noqa: F401  (loads libc10/libtorch for the extension)
        _MOD = _Counted(importlib.import_module("lumenrl_b200._C"))
    except Exception as e:  # pragma: no cover - depends on the build
        _ERR = e


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
