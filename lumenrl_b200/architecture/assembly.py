"""Build the runtime component graph from config.

Backends accepted: training ``fsdp``/``fsdp2`` (this framework's sharded
trainer) and ``megatron``/``megatron_native`` (its tensor/expert/pipeline
parallel engine); inference ``native`` plus the reference's names ``atom``
and ``vllm``, which resolve to the native engine.  The trainer follows the
algorithm (``opd`` -> OPD, ``spec_distill`` -> speculative distillation,
``async_training.enabled`` -> async, else the synchronous RL trainer).
"""

from __future__ import annotations

from dataclasses import dataclass

from lumenrl_b200.architecture.registries import (inference_backend_registry, trainer_registry,
                                                  training_backend_registry, worker_role_registry)

ALLOWED_TRAINING = {"fsdp", "fsdp2", "megatron", "megatron_native"}
ALLOWED_INFERENCE = {"native", "atom", "vllm"}


def validate_backend_policy(cfg) -> None:
    if cfg.training_backend not in ALLOWED_TRAINING:
        raise ValueError(f"Training backend must be one of {sorted(ALLOWED_TRAINING)}")
    if cfg.inference_backend not in ALLOWED_INFERENCE:
        raise ValueError(f"Inference backend must be one of {sorted(ALLOWED_INFERENCE)}")


def _ensure(reg, key, value) -> None:
    if key not in reg:
        reg.register(key, value)


def register_default_bindings() -> None:
    from lumenrl_b200.engine.inference.engine import RolloutEngine
    from lumenrl_b200.engine.training.actor import ActorEngine
    from lumenrl_b200.trainer.async_trainer import AsyncRLTrainer
    from lumenrl_b200.trainer.opd_trainer import OPDTrainer
    from lumenrl_b200.trainer.rl_trainer import RLTrainer
    from lumenrl_b200.trainer.sft_trainer import SFTTrainer
    from lumenrl_b200.trainer.spec_distill_trainer import SpecDistillTrainer
    from lumenrl_b200.workers import roles
    for key, cls in {"actor.default": roles.ActorWorker, "critic.default": roles.CriticWorker,
                     "ref.default": roles.RefWorker, "reward.default": roles.RewardWorker,
                     "rollout.native": roles.RolloutWorker, "rollout.atom": roles.RolloutWorker,
                     "rollout.vllm": roles.RolloutWorker, "teacher.default": roles.TeacherWorker,
                     "hybrid.default": roles.HybridWorker}.items():
        _ensure(worker_role_registry, key, cls)
    for key in ("fsdp", "fsdp2", "megatron", "megatron_native"):
        _ensure(training_backend_registry, key, ActorEngine)
    for key in ("native", "atom", "vllm"):
        _ensure(inference_backend_registry, key, RolloutEngine)
    _ensure(trainer_registry, "trainer.rl", RLTrainer)
    _ensure(trainer_registry, "trainer.async", AsyncRLTrainer)
    _ensure(trainer_registry, "trainer.opd", OPDTrainer)
    _ensure(trainer_registry, "trainer.spec_distill", SpecDistillTrainer)
    _ensure(trainer_registry, "trainer.sft", SFTTrainer)


@dataclass
class RuntimeGraph:
    actor_worker_cls: type
    rollout_worker_cls: type
    trainer_cls: type
    training_backend_cls: type
    inference_backend_cls: type


class RuntimeAssembler:
    def __init__(self, config) -> None:
        self.config = config
        register_default_bindings()

    def _trainer_key(self) -> str:
        algo = self.config.algorithm.name.lower()
        if algo == "opd":
            return "trainer.opd"
        if algo == "spec_distill":
            return "trainer.spec_distill"
        if algo == "sft":
            return "trainer.sft"
        if self.config.async_training.enabled:
            return "trainer.async"
        return "trainer.rl"

    def build_graph(self) -> dict[str, type]:
        a = self.config.assembly
        if a.strict_policy:
            validate_backend_policy(a)
        g = RuntimeGraph(
            actor_worker_cls=worker_role_registry.get(a.role_impl_keys.get("actor", "actor.default")),
            rollout_worker_cls=worker_role_registry.get(a.role_impl_keys.get("rollout", f"rollout.{a.inference_backend}")),
            trainer_cls=trainer_registry.get(self._trainer_key()),
            training_backend_cls=training_backend_registry.get(a.training_backend),
            inference_backend_cls=inference_backend_registry.get(a.inference_backend))
        return dict(g.__dict__)
