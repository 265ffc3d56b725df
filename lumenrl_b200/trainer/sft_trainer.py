"""Supervised fine-tuning with the same engines
(reference ``lumenrl/trainer/sft_trainer.py:41-271``).

Rows are (prompt, response) token pairs; the loss is the NLL of the response
tokens (optionally the ``loss_mask`` of a chat-templated conversation), with
the token-mean over the global batch (``sft_loss`` conventions), packed
micro-batches and the sharded AdamW.
"""

from __future__ import annotations

import time
from typing import Optional

import torch

from lumenrl_b200.core.protocol import DataProto
from lumenrl_b200.engine.training.actor import ActorEngine
from lumenrl_b200.engine.training.packing import make_micro_batches, pack_from_grid
from lumenrl_b200.models.config import ModelArgs
from lumenrl_b200.parallel.dist import ParallelState, all_reduce_sum


class SFTTrainer:
    def __init__(self, config, model_args: ModelArgs, state: ParallelState) -> None:
        from lumenrl_b200.ops.kernel_flags import apply_kernels_config
        apply_kernels_config(getattr(config, "kernels", None))
        p = config.policy
        self.config = config
        from lumenrl_b200.engine.training.fsdp import ShardedParamActorEngine, wants_param_sharding
        # SFT has no rollout engine sharing the weights, so FSDP2-style full
        # sharding (policy.training.fsdp_cfg.reshard_after_forward) is honoured
        engine_cls = ShardedParamActorEngine if wants_param_sharding(config) else ActorEngine
        self.engine = engine_cls(model_args, state, lr=p.learning_rate, weight_decay=p.weight_decay,
                                  max_grad_norm=p.max_grad_norm, seed=config.seed,
                                  total_steps=config.num_training_steps, warmup_steps=p.lr_warmup_steps,
                                  lr_style=p.lr_decay_style)
        self.state = state
        self.global_step = 0

    def step(self, batch: DataProto) -> dict:
        t = batch.tensors
        dev = self.state.device
        mask = t.get("loss_mask", t["response_mask"]).float()
        cp = self.engine.cp
        # the ranks of a context-parallel group hold the same rows: count them once
        total = max(all_reduce_sum(float(mask.sum()), self.state) / cp, 1.0)
        lens = (t["prompt_lengths"] + t["response_lengths"]).tolist()
        nll = 0.0
        t0 = time.perf_counter()
        for rows in make_micro_batches(lens, rows_per_micro=self.config.policy.train_micro_batch_size):
            pb = pack_from_grid(t["prompt_ids"], t["prompt_lengths"], t["responses"], t["response_lengths"], rows, dev,
                                cp, self.engine.cp_rank)
            lp, _ = self.engine._forward_scored(pb, 1.0, want_entropy=False)
            r_idx = torch.as_tensor(rows, device=dev)[pb.out_row]
            w = mask[r_idx, pb.out_col]
            loss = -(lp * w).sum() / total
            loss.backward()
            nll += float(loss.detach())
        st = self.engine.opt.step(self.engine.sched.current if self.engine.sched else None)
        if self.engine.sched:
            self.engine.sched.step()
        self.global_step += 1
        return {"sft/loss": nll, "sft/grad_norm": st["grad_norm"], "sft/step_s": time.perf_counter() - t0,
                "step": self.global_step}
