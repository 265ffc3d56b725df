"""verl plugin entry point (reference ``lumenrl/plugin/verl/register.py:26-264``,
``atom_replica.py:20-164``; entry point ``pyproject.toml:45-46``).

``register()`` adds this framework's in-process rollout engine to verl's
rollout registry under ``"lumenrl_b200"`` when verl is importable; it always
records the adapters in ``PLUGIN_REGISTRY`` so the same classes can be found
without verl.  Unlike the reference's ATOM adapter, the rollout adapter here
implements generation itself (the engine runs in the worker's process on the
actor's weights), and ``update_weights`` loads the streamed named tensors.
"""

from __future__ import annotations

import logging
from typing import Any, Iterable

logger = logging.getLogger(__name__)

PLUGIN_REGISTRY: dict[str, str] = {}
_registered = False


class RolloutAdapter:
    """verl ``BaseRollout``-shaped wrapper around ``RolloutEngine``."""

    def __init__(self, config: Any = None, model_config: Any = None, device_mesh: Any = None, engine: Any = None,
                 **kw: Any) -> None:
        try:  # keep verl's bookkeeping when it is present
            from verl.workers.rollout.base import BaseRollout
            BaseRollout.__init__(self, config, model_config, device_mesh)
        except Exception:  # noqa: BLE001 - verl absent or a different version
            pass
        self.engine = engine
        self.config = config

    def set_engine(self, engine: Any) -> None:
        self.engine = engine

    async def resume(self, tags: list = None) -> None:
        if self.engine is not None:
            self.engine.wake()

    async def release(self) -> None:
        if self.engine is not None:
            self.engine.sleep()

    async def update_weights(self, weights: Iterable, wire_format: str = "named_tensors", **kw: Any) -> None:
        """Copy HF-named tensors into the engine's weights (no-op when the
        engine shares the actor's buffer, i.e. colocated)."""
        if self.engine is None:
            return
        sd = dict(weights)
        if sd:
            self.engine.model.load_hf_state_dict(sd, strict=False)
        self.engine.update_weights()

    def generate_sequences(self, prompts: list, n: int = 1, max_new_tokens: int = 1024, temperature: float = 1.0,
                           seed: int = 0) -> Any:
        from lumenrl_b200.engine.inference.engine import SamplingParams
        return self.engine.generate(prompts, SamplingParams(max_new_tokens=max_new_tokens, temperature=temperature,
                                                            n=n, seed=seed))


def register() -> bool:
    """Entry point for ``verl.plugins``; True if verl's registry was updated."""
    global _registered
    PLUGIN_REGISTRY["rollout:lumenrl_b200"] = f"{__name__}.RolloutAdapter"
    PLUGIN_REGISTRY["trainer:lumenrl_b200_grpo"] = "lumenrl_b200.trainer.rl_trainer.RLTrainer"
    if _registered:
        return True
    try:
        from verl.workers.rollout import base as vbase  # type: ignore
    except Exception:  # noqa: BLE001
        logger.info("lumenrl_b200: verl not importable; adapters kept in PLUGIN_REGISTRY only")
        return False
    reg = getattr(vbase, "_ROLLOUT_REGISTRY", None)
    if isinstance(reg, dict):
        reg[("lumenrl_b200", "async")] = f"{__name__}.RolloutAdapter"
        _registered = True
    return _registered
