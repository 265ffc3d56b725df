"""Command-line entry point (reference ``lumenrl/trainer/main.py:57-144``).

    torchrun --nproc-per-node 8 -m lumenrl_b200.trainer.main --config configs/grpo_qwen3_8b.yaml \
        algorithm.grpo.num_generations=8 num_training_steps=100

Loads the YAML (+ dot-list overrides), joins the process group (NCCL on GPU,
gloo on CPU; short timeout), resolves the trainer through the runtime
assembler, attaches logging / checkpoint / W&B callbacks and trains.
Synthetic-workload knobs (prompt length, prompts per step, reward) come from
``--prompt-len`` etc. or default to the policy section of the config.
"""

from __future__ import annotations

import argparse
import logging
import os
import sys


def _setup_logging() -> None:
    level = os.environ.get("LUMENRL_LOG_LEVEL", "INFO").upper()
    rank = int(os.environ.get("RANK", "0"))
    logging.basicConfig(level=level if rank == 0 else "WARNING", stream=sys.stdout,
                        format="%(asctime)s %(levelname)s %(name)s: %(message)s")


def main(argv=None) -> list:
    _setup_logging()
    ap = argparse.ArgumentParser(description="lumenrl_b200 trainer")
    ap.add_argument("--config", required=True)
    ap.add_argument("--prompt-len", type=int, default=None)
    ap.add_argument("--prompts-per-step", type=int, default=None)
    ap.add_argument("--reward", default=None)
    args, overrides = ap.parse_known_args(argv)
    from lumenrl_b200.architecture.assembly import RuntimeAssembler
    from lumenrl_b200.core.config import LumenRLConfig
    from lumenrl_b200.models.config import resolve_model
    from lumenrl_b200.parallel.dist import init_distributed
    from lumenrl_b200.trainer.callbacks import CheckpointCallback, LoggingCallback, WandbCallback
    from lumenrl_b200.trainer.rl_trainer import RLRunSpec
    cfg = LumenRLConfig.from_yaml(args.config, overrides)
    st = init_distributed(timeout_s=float(os.environ.get("NCCL_TIMEOUT", 1800)))
    cfg.assembly.strict_policy = True
    graph = RuntimeAssembler(cfg).build_graph()
    p = cfg.policy
    algo = getattr(cfg.algorithm, cfg.algorithm.name, cfg.algorithm.grpo)
    group = int(getattr(algo, "num_generations", 1) or 1)
    prompts = args.prompts_per_step or max(1, p.train_global_batch_size // max(group, 1))
    max_new = min(p.max_response_length, max(1, p.max_total_sequence_length - (args.prompt_len or 512)))
    spec = RLRunSpec(prompts_per_step=prompts, prompt_len=args.prompt_len or 512, prompt_low=3,
                     prompt_high=resolve_model(p.model_name or "tiny-llama").vocab_size, max_new_tokens=max_new,
                     reward=args.reward or cfg.reward.function, rows_per_micro=p.train_micro_batch_size)
    trainer = graph["trainer_cls"](cfg, resolve_model(p.model_name or "tiny-llama"), spec, st).setup()
    trainer.callbacks = [LoggingCallback(cfg.logger.log_interval),
                         CheckpointCallback(cfg.checkpointing.checkpoint_dir, cfg.checkpointing.save_steps,
                                            cfg.checkpointing.save_total_limit)]
    if cfg.logger.wandb_enabled:
        trainer.callbacks.append(WandbCallback(cfg.logger.wandb.project, cfg.logger.wandb.name, cfg.logger.wandb.entity))
    hist = trainer.train()
    trainer.cleanup()
    return hist


if __name__ == "__main__":
    main()
