"""Trainer callbacks (reference ``lumenrl/trainer/callbacks.py:23-391``):
logging, periodic checkpointing with pruning and a latest-step tracker,
periodic evaluation, and a Weights & Biases logger that degrades to a JSONL
file when ``wandb`` is not installed."""

from __future__ import annotations

import json
import logging
import os
import time

logger = logging.getLogger(__name__)


class Callback:
    def on_train_begin(self, trainer) -> None: ...
    def on_step_end(self, trainer, metrics: dict) -> None: ...
    def on_train_end(self, trainer) -> None: ...


class LoggingCallback(Callback):
    def __init__(self, interval: int = 1, keys: tuple = ("reward/mean", "actor/pg_loss", "actor/grad_norm",
                                                          "perf/step_tokens_per_s", "timing/step_s")) -> None:
        self.interval, self.keys = interval, keys

    def on_step_end(self, trainer, m: dict) -> None:
        if m.get("step", 0) % self.interval == 0 and getattr(trainer.state, "rank", 0) == 0:
            logger.info("step %s | %s", m.get("step"), " ".join(f"{k}={m[k]:.4g}" for k in self.keys if k in m))


class CheckpointCallback(Callback):
    def __init__(self, root: str, save_steps: int = 50, save_total_limit: int = 3) -> None:
        from lumenrl_b200.utils.checkpoint import CheckpointManager
        self.mgr = CheckpointManager(root, save_total_limit)
        self.save_steps = save_steps

    def on_step_end(self, trainer, m: dict) -> None:
        step = int(m.get("step", 0))
        if self.save_steps > 0 and step % self.save_steps == 0:
            st = trainer.state
            self.mgr.save(trainer.actor, step, st.rank, st.world_size, {"data": trainer.data.state_dict()})

    def on_train_begin(self, trainer) -> None:
        st = trainer.state
        step = self.mgr.load_latest(trainer.actor, st.rank, st.world_size, data=getattr(trainer, "data", None))
        if step:
            trainer.global_step = step
            logger.info("resumed from step %d", step)


class EvalCallback(Callback):
    def __init__(self, fn, interval: int = 1000) -> None:
        self.fn, self.interval = fn, interval

    def on_step_end(self, trainer, m: dict) -> None:
        if self.interval > 0 and int(m.get("step", 0)) % self.interval == 0:
            m.update(self.fn(trainer))


class WandbCallback(Callback):
    def __init__(self, project: str = "lumenrl", name: str = "", entity=None, fallback_dir: str = "outputs") -> None:
        self.run = None
        try:
            import wandb  # noqa: F401
            self.run = wandb.init(project=project, name=name or None, entity=entity)
        except Exception:
            os.makedirs(fallback_dir, exist_ok=True)
            self.path = os.path.join(fallback_dir, f"metrics_{int(time.time())}.jsonl")

    def on_step_end(self, trainer, m: dict) -> None:
        from lumenrl_b200.trainer.metrics import with_aliases
        mm = with_aliases(m)
        if self.run is not None:
            self.run.log(mm, step=int(m.get("step", 0)))
        elif getattr(trainer.state, "rank", 0) == 0:
            with open(self.path, "a") as f:
                f.write(json.dumps({k: v for k, v in mm.items() if isinstance(v, (int, float))}) + "\n")
