"""Frozen teacher LM head rebuilt from safetensors shards
(reference ``lumenrl/core/teacher_lm_head.py:22-119``).

Loads only ``lm_head.weight`` (and optionally the final norm weight) from a
checkpoint directory, without instantiating the teacher, and turns teacher
hidden states into logits: ``logits = RMSNorm(h) @ W^T``.  Used by OPD and
speculative-decoding distillation where the teacher's hidden states come from
another process or GPU.
"""

from __future__ import annotations

import json
import os
from typing import Optional

import torch
from torch import Tensor

from lumenrl_b200 import ops


class TeacherLMHead:
    def __init__(self, weight: Tensor, norm_weight: Optional[Tensor] = None, eps: float = 1e-6) -> None:
        self.weight = weight
        self.norm_weight = norm_weight
        self.eps = eps

    @classmethod
    def from_pretrained(cls, path: str, lm_head_key: str = "lm_head.weight", norm_key: str = "model.norm.weight",
                        load_norm: bool = False, device="cpu", dtype=torch.bfloat16, eps: float = 1e-6):
        from safetensors import safe_open
        idx = os.path.join(path, "model.safetensors.index.json")
        if os.path.isfile(idx):
            with open(idx) as f:
                wmap = json.load(f)["weight_map"]
        else:
            wmap = {}
            for n in os.listdir(path):
                if n.endswith(".safetensors"):
                    with safe_open(os.path.join(path, n), "pt") as f:
                        for k in f.keys():
                            wmap[k] = n

        def get(key: str) -> Tensor:
            if key not in wmap:
                alt = "model.embed_tokens.weight" if key == lm_head_key else None
                if alt is None or alt not in wmap:
                    raise KeyError(f"{key} not found under {path}")
                key = alt           # tied embeddings
            with safe_open(os.path.join(path, wmap[key]), "pt") as f:
                return f.get_tensor(key).to(device=device, dtype=dtype)
        w = get(lm_head_key)
        nw = get(norm_key) if load_norm else None
        return cls(w, nw, eps)

    def logits(self, hidden: Tensor) -> Tensor:
        h = ops.rmsnorm(hidden, self.norm_weight, self.eps) if self.norm_weight is not None else hidden
        return h.to(self.weight.dtype) @ self.weight.t()

    __call__ = logits
