"""Runtime assembly: typed registries and the assembler that resolves the
trainer, worker roles and backends from config (reference
``lumenrl/architecture/assembly/runtime_assembler.py:27-59``)."""

from lumenrl_b200.architecture.assembly import RuntimeAssembler, validate_backend_policy  # noqa: F401
from lumenrl_b200.architecture.registries import (  # noqa: F401
    inference_backend_registry, trainer_registry, training_backend_registry, worker_role_registry,
)
