"""Expert-weight routing between the HF spellings of an MoE layer and the
native layout, with a sync-coverage check (reference:
``lumenrl/engine/inference/vllm_moe_weight_sync.py:1-365``, which maps HF
fused 3D expert tensors onto vLLM's ``w13_weight`` / ``w2_weight`` and
asserts that a sync covers every parameter).

HF spells a layer's experts two ways:

- per expert (safetensors checkpoints): ``<p>.experts.<e>.gate_proj.weight``
  [F, H], ``<p>.experts.<e>.up_proj.weight`` [F, H],
  ``<p>.experts.<e>.down_proj.weight`` [H, F];
- fused (``transformers`` >= 5 modules): ``<p>.experts.gate_up_proj``
  [E, 2F, H] with the gate rows first, ``<p>.experts.down_proj`` [E, H, F].

The native MoE layer keeps exactly the fused layout (``experts_w13``
[E, 2F, H], ``experts_w2`` [E, H, F]), so splitting is views and fusing is one
stack per tensor.  ``route_expert_weights`` converts a state dict to whichever
spelling the receiving module uses.
"""

from __future__ import annotations

import re
from typing import Iterable

import torch
from torch import Tensor

_PER = re.compile(r"^(.*)\.experts\.(\d+)\.(gate_proj|up_proj|down_proj)\.weight$")
_FUSED = re.compile(r"^(.*)\.experts\.(gate_up_proj|down_proj)$")


def split_experts(sd: dict[str, Tensor]) -> dict[str, Tensor]:
    """Fused expert tensors -> per-expert views; every other entry unchanged."""
    out: dict[str, Tensor] = {}
    for k, v in sd.items():
        m = _FUSED.match(k)
        if m is None:
            out[k] = v
            continue
        p, kind = m.group(1), m.group(2)
        if v.dim() != 3:
            raise ValueError(f"{k}: fused expert tensor must be 3-D, got {tuple(v.shape)}")
        for e in range(v.shape[0]):
            if kind == "gate_up_proj":
                if v.shape[1] % 2:
                    raise ValueError(f"{k}: odd gate/up row count {v.shape[1]}")
                F = v.shape[1] // 2
                out[f"{p}.experts.{e}.gate_proj.weight"] = v[e, :F]
                out[f"{p}.experts.{e}.up_proj.weight"] = v[e, F:]
            else:
                out[f"{p}.experts.{e}.down_proj.weight"] = v[e]
    return out


def fuse_experts(sd: dict[str, Tensor]) -> dict[str, Tensor]:
    """Per-expert tensors -> fused [E, 2F, H] / [E, H, F] stacks.  Experts of
    a layer must be numbered 0..E-1 with all three matrices present."""
    out: dict[str, Tensor] = {}
    layers: dict[str, dict[int, dict[str, Tensor]]] = {}
    for k, v in sd.items():
        m = _PER.match(k)
        if m is None:
            out[k] = v
            continue
        layers.setdefault(m.group(1), {}).setdefault(int(m.group(2)), {})[m.group(3)] = v
    for p, experts in layers.items():
        E = len(experts)
        if sorted(experts) != list(range(E)):
            raise KeyError(f"{p}: experts {sorted(experts)[:8]} are not numbered 0..{E - 1}")
        for e, mats in experts.items():
            absent = {"gate_proj", "up_proj", "down_proj"} - set(mats)
            if absent:
                raise KeyError(f"{p}.experts.{e}: missing {sorted(absent)}")
        out[f"{p}.experts.gate_up_proj"] = torch.stack(
            [torch.cat([experts[e]["gate_proj"], experts[e]["up_proj"]], 0) for e in range(E)])
        out[f"{p}.experts.down_proj"] = torch.stack([experts[e]["down_proj"] for e in range(E)])
    return out


def route_expert_weights(sd: dict[str, Tensor], target_names: Iterable[str]) -> dict[str, Tensor]:
    """``sd`` in the expert spelling the receiver uses: fused when the target
    has any fused expert parameter, per-expert otherwise."""
    names = set(target_names)
    wants_fused = any(_FUSED.match(n) for n in names)
    has_fused = any(_FUSED.match(k) for k in sd)
    has_per = any(_PER.match(k) for k in sd)
    if wants_fused and has_per:
        return fuse_experts(sd)
    if not wants_fused and has_fused:
        return split_experts(sd)
    return sd


def assert_weight_sync_coverage(sd: dict[str, Tensor], target_shapes: dict[str, tuple],
                                optional: Iterable[str] = ()) -> None:
    """Raise ``KeyError`` unless ``sd`` covers every target parameter (except
    ``optional`` ones, e.g. a tied LM head), brings no tensor that matches no
    parameter, and agrees with every parameter's shape."""
    opt = set(optional)
    missing = [k for k in target_shapes if k not in sd and k not in opt]
    extra = [k for k in sd if k not in target_shapes and k not in opt]
    bad = [k for k, v in sd.items() if k in target_shapes and tuple(v.shape) != tuple(target_shapes[k])]
    if missing or extra or bad:
        raise KeyError(f"weight sync coverage: missing {missing[:6]}, unexpected {extra[:6]}, "
                       f"shape mismatch {bad[:6]}")
