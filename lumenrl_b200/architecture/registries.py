"""Typed component registries used by the runtime assembler."""

from lumenrl_b200.core.registry import Registry

worker_role_registry = Registry("worker_role")
training_backend_registry = Registry("training_backend")
inference_backend_registry = Registry("inference_backend")
trainer_registry = Registry("trainer")
