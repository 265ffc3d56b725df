"""Colocated (fused) worker classes: several roles in one process.

``create_colocated_worker_cls({"actor": A, "ref": R})`` builds a class whose
instances hold one instance per role and expose every public method of role
``x`` as ``x_<method>`` (reference ``lumenrl/controller/colocation.py:11-61``).
Together with ``WorkerGroup.spawn`` this lets actor, reference and rollout
share GPUs and memory.
"""

from __future__ import annotations

from typing import Any


def create_colocated_worker_cls(role_classes: dict[str, type], role_kwargs: dict[str, dict] | None = None) -> type:
    role_kwargs = role_kwargs or {}

    def __init__(self, *args: Any, **kwargs: Any) -> None:
        self._roles = {}
        for role, cls in role_classes.items():
            self._roles[role] = cls(*args, **{**kwargs, **role_kwargs.get(role, {})})

    def __getattr__(self, name: str):
        roles = object.__getattribute__(self, "_roles")
        for role, inst in roles.items():
            pre = role + "_"
            if name.startswith(pre):
                return getattr(inst, name[len(pre):])
        raise AttributeError(name)

    def role(self, name: str):
        return self._roles[name]

    return type("Colocated_" + "_".join(role_classes), (object,), {"__init__": __init__, "__getattr__": __getattr__,
                                                                    "role": role})


def worker_class_for(role_key: str):
    """Resolve a registered worker role key to its class (reference
    ``controller/worker_group_factory.py:9-12``)."""
    from lumenrl_b200.core.registry import WORKER_REGISTRY
    import lumenrl_b200.workers  # noqa: F401  (registers the roles)
    return WORKER_REGISTRY.get(role_key)


resolve_worker_class = worker_class_for
