"""Kernel and collective selection from the config's ``kernels`` section.

Every switch also exists as an ``LRL_*`` environment variable (read once at
import by the modules that own the switch, or at call time by the
collectives).  ``apply_kernels_config`` makes a config value win over both:
it rewrites the owning module's switch and the environment variable, so later
imports and spawned ranks see the same choice.  ``None`` fields change
nothing.
"""

from __future__ import annotations

import importlib
import os
from typing import Any

# config field -> (environment variable, owning module, module attribute,
#                  allowed values; None = boolean)
_FLAGS = {
    "train_gemm": ("LRL_TRAIN_GEMM", "lumenrl_b200.ops", "TRAIN_GEMM", ("own", "cublas")),
    "train_attn": ("LRL_TRAIN_ATTN", "lumenrl_b200.ops.attention", "TRAIN_ATTN", ("tc", "fa2")),
    "train_attn_bwd": ("LRL_TRAIN_ATTN_BWD", "lumenrl_b200.ops.attention", "TRAIN_ATTN_BWD", ("tc", "fa2")),
    "decode_gemm": ("LRL_DECODE_GEMM", "lumenrl_b200.ops", "DECODE_GEMM", ("auto", "sk", "skinny", "cublas")),
    "fp8_decode_gemm": ("LRL_FP8_DECODE_GEMM", "lumenrl_b200.ops", "FP8_DECODE_GEMM", ("stream", "gemm")),
    "decode_attn": ("LRL_DECODE_ATTN", "lumenrl_b200.ops", "DECODE_ATTN", ("tma", "cp")),
    "nvls": ("LRL_NVLS", None, None, None),
    "cp_ring": ("LRL_CP_RING", None, None, ("nvlink", "pg")),
    "draft_allreduce": ("LRL_DRAFT_ALLREDUCE", None, None, ("nvlink", "nccl")),
    "debug_bounds": ("LRL_DEBUG_BOUNDS", None, None, None),
    "eagle_kernels": ("LRL_EAGLE_KERNELS", "lumenrl_b200.models.eagle3", "_KERNELS", None),
}


def apply_kernels_config(kernels: Any) -> dict[str, str]:
    """Apply the non-None fields of ``kernels`` (a ``KernelsConfig``);
    returns {environment variable: value} of what was set."""
    applied: dict[str, str] = {}
    if kernels is None:
        return applied
    for name, (env, module, attr, allowed) in _FLAGS.items():
        val = getattr(kernels, name, None)
        if val is None:
            continue
        if allowed is None:
            flag = bool(val) if isinstance(val, bool) else str(val).lower() in ("1", "true", "yes", "on")
            text = "1" if flag else "0"
            mod_val: Any = flag
        else:
            text = str(val).lower()
            if text not in allowed:
                raise ValueError(f"kernels.{name}={val!r}: expected one of {allowed}")
            mod_val = text
        os.environ[env] = text
        applied[env] = text
        if module is not None:
            setattr(importlib.import_module(module), attr, mod_val)
        if name == "debug_bounds":
            # the extension proxy picks the checked comm module on its next load
            ext_mod = importlib.import_module("lumenrl_b200.ops.ext")
            if ext_mod._MOD is not None and bool(ext_mod._MOD._bounds is not None) != mod_val:
                ext_mod._MOD, ext_mod._ERR = None, None
    return applied
