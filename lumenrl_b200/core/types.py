"""Enumerations shared across the framework (reference ``lumenrl/core/types.py:8-24``).

``GenerationBackend`` adds ``native``: this framework's own rollout engine.
The reference names ``atom``/``vllm`` are accepted and mapped to it.
"""

from __future__ import annotations

from enum import Enum


class TrainingBackend(str, Enum):
    FSDP2 = "fsdp2"
    MEGATRON_NATIVE = "megatron_native"
    NONE = "none"


class GenerationBackend(str, Enum):
    NATIVE = "native"
    ATOM = "atom"
    VLLM = "vllm"


class AlgorithmName(str, Enum):
    GRPO = "grpo"
    DAPO = "dapo"
    PPO = "ppo"
    OPD = "opd"
    SPEC_DISTILL = "spec_distill"
