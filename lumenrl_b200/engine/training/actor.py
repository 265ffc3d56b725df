"""Training engine for the policy (and reference / critic) model.

Replaces the reference's FSDP2 engine + actor worker hot path
(``lumenrl/engine/training/fsdp_engine.py:63-722``,
``lumenrl/workers/actor_worker.py:290-792``):

* ``compute_log_probs``: no-grad packed forward in token-budget micro
  batches, fused LM-head log-prob (+ entropy), scattered to ``[B, R]``.
* ``update_policy``: for each mini-batch and PPO epoch, packed forward with
  grad per micro-batch, the clipped-ratio loss on the flat stream of scored
  tokens (one fused kernel), backward accumulating fp32 ``main_grad``, then
  one sharded AdamW step.  Loss normalisation is the global token mean
  (``token-mean``): each rank divides its token sum by the token count of the
  whole mini-batch over all ranks, and gradients are SUM-reduced.
* Activation recomputation per decoder layer is on when
  ``policy.training.megatron_cfg.recompute_granularity`` or HF
  gradient-checkpointing asks for it (``gradient_checkpointing=True``).
"""

from __future__ import annotations

import logging
import math
import time
from typing import Any, Optional

import torch
from torch import Tensor

from lumenrl_b200 import ops
from lumenrl_b200.core.protocol import DataProto
from lumenrl_b200.engine.training.lr_scheduler import LRSchedule
from lumenrl_b200.engine.training.optimizer import ShardedFlatAdamW
from lumenrl_b200.engine.training.packing import PackedBatch, make_micro_batches, pack_from_grid
from lumenrl_b200.models.config import ModelArgs
from lumenrl_b200.models.qwen3 import FlatLayout, Qwen3Model, param_specs
from lumenrl_b200.parallel.dist import ParallelState, all_reduce_sum

logger = logging.getLogger(__name__)


def padded_numel(args: ModelArgs, world: int) -> int:
    n = FlatLayout(param_specs(args)).numel
    q = world * 128
    return (n + q - 1) // q * q


class ActorEngine:
    def __init__(self, args: ModelArgs, state: ParallelState, *, lr: float = 1e-6, betas=(0.9, 0.999),
                 eps: float = 1e-8, weight_decay: float = 0.01, max_grad_norm: float = 1.0, seed: int = 0,
                 dtype: Optional[torch.dtype] = None, trainable: bool = True, gradient_checkpointing: bool = False,
                 total_steps: int = 1000, warmup_steps: int = 0, lr_style: str = "constant", min_lr_ratio: float = 0.0,
                 comm=None, init: bool = True, fused_comm: bool = True) -> None:
        self.args = args
        self.state = state
        self.device = state.device
        if dtype is None:
            dtype = torch.bfloat16 if self.device.type == "cuda" else torch.float32
        numel = padded_numel(args, state.world_size if trainable else 1)
        if comm is None and trainable and state.world_size > 1 and self.device.type == "cuda" and fused_comm:
            from lumenrl_b200.parallel.symm import NVLinkOptimizerComm
            comm = NVLinkOptimizerComm(numel, state.rank, state.world_size, dtype, group=state.dp_group)
        if comm is not None and hasattr(comm, "weights"):
            flat = comm.weights.tensor      # resident weights live in NVLink-mapped memory
        else:
            flat = torch.zeros(numel, dtype=dtype, device=self.device)
        self.comm = comm
        self.model = Qwen3Model(args, device=self.device, dtype=dtype, flat=flat, requires_grad=trainable)
        if init:
            self.model.init_weights(seed)
        self.model.gradient_checkpointing = gradient_checkpointing is True
        self.recompute_policy = "auto" if gradient_checkpointing == "auto" else None
        # context parallelism: this rank scores its zigzag share of every
        # sequence; the optimizer still reduces over all ranks (a CP group's
        # ranks hold the same rows, so they add up like data-parallel ranks)
        self.cp, self.cp_rank, self.cp_group = state.cp_size, state.cp_rank, state.cp_group
        if self.cp > 1:
            self.model.cp_group = state.cp_group
        self.trainable = trainable
        self.opt: Optional[ShardedFlatAdamW] = None
        self.sched: Optional[LRSchedule] = None
        if trainable:
            self.opt = ShardedFlatAdamW(flat, state.world_size, state.rank, lr=lr, betas=betas, eps=eps,
                                        weight_decay=weight_decay, max_grad_norm=max_grad_norm, comm=comm,
                                        group=state.dp_group)
            self.model.attach_main_grad(self.opt.grad)
            self.sched = LRSchedule(lr, total_steps, warmup_steps, lr_style, min_lr_ratio)

    # ------------------------------------------------------------------ scoring
    def _forward_scored(self, pb: PackedBatch, temperature: float, want_entropy: bool):
        h = self.model.forward_packed(pb.input_ids, pb.positions, pb.cu_seqlens, pb.max_seqlen)
        hs = h.index_select(0, pb.score_index)
        return ops.token_logprob(hs, self.model.lm_head, pb.targets, temperature=temperature,
                                 want_entropy=want_entropy)

    @torch.no_grad()
    def compute_log_probs(self, batch: DataProto, temperature: float = 1.0, token_budget: int = 16384,
                          want_entropy: bool = True) -> tuple[Tensor, Optional[Tensor]]:
        t = batch.tensors
        B, R = t["responses"].shape
        lens = (t["prompt_lengths"] + t["response_lengths"]).tolist()
        logp = torch.zeros(B, R, dtype=torch.float32, device=self.device)
        ent = torch.zeros(B, R, dtype=torch.float32, device=self.device) if want_entropy else None
        pl_h, rl_h = t["prompt_lengths"].tolist(), t["response_lengths"].tolist()
        for rows in make_micro_batches(lens, token_budget=token_budget):
            pb = pack_from_grid(t["prompt_ids"], pl_h, t["responses"], rl_h, rows, self.device, self.cp, self.cp_rank)
            self._set_replay(batch, pb)
            lp, e = self._forward_scored(pb, temperature, want_entropy)
            rows_t = torch.as_tensor(rows, device=self.device)[pb.out_row]
            logp[rows_t, pb.out_col] = lp
            if want_entropy:
                ent[rows_t, pb.out_col] = e
        self.model.routing_replay = None
        if self.cp > 1:   # each CP rank scored its own positions; the others are zero
            torch.distributed.all_reduce(logp, group=self.cp_group)
            if want_entropy:
                torch.distributed.all_reduce(ent, group=self.cp_group)
        return logp, ent

    def _set_replay(self, batch: DataProto, pb: PackedBatch) -> None:
        if self.args.num_experts == 0 or "routed_experts" not in batch.ragged:
            self.model.routing_replay = None
            return
        from lumenrl_b200.moe.r3 import RoutingReplay
        self.model.routing_replay = RoutingReplay.from_rows(
            [batch.ragged["routed_experts"][r] for r in pb.rows],
            (pb.cu_seqlens[1:] - pb.cu_seqlens[:-1]).tolist(), self.args, self.device)

    # ------------------------------------------------------------------ training
    def update_policy(self, batch: DataProto, algo_cfg, algorithm: str = "grpo", rows_per_micro: int = 4,
                      token_budget: int = 0, num_mini_batches: int = 1, num_epochs: int = 1,
                      temperature: float = 1.0) -> dict[str, float]:
        assert self.opt is not None
        t = batch.tensors
        B = t["responses"].shape[0]
        lens = (t["prompt_lengths"] + t["response_lengths"]).tolist()
        mask_grid = t["response_mask"].float()
        if "dapo_sample_mask" in t:
            mask_grid = mask_grid * t["dapo_sample_mask"].float().reshape(-1, 1)
        metrics: dict[str, float] = {}
        rstats = getattr(self.model, "router_stats", None)
        if rstats is None and self.args.num_experts:
            from lumenrl_b200.moe.diagnostics import attach_router_stats
            rstats = attach_router_stats(self.model, self.device)
        if rstats is not None:
            rstats.reset()
        if self.recompute_policy == "auto" and self.device.type == "cuda":
            rows = rows_per_micro or B
            tok = max(sum(sorted(lens, reverse=True)[:rows]), 1)
            metrics["actor/recompute_layers"] = float(self.plan_recompute(tok))
        # per-micro-batch statistics stay on the device until the end
        sums: dict = {"pg_loss": 0.0, "ppo_kl": 0.0, "clipfrac": 0.0, "tok": 0.0, "entropy": 0.0}
        lens_h = (t["prompt_lengths"].tolist(), t["response_lengths"].tolist())
        t_fwd_bwd = 0.0
        opt_stats = {}
        opt_t = {"opt_rs_s": 0.0, "opt_bcast_s": 0.0}
        for _epoch in range(num_epochs):
            mini_size = math.ceil(B / num_mini_batches)
            for m0 in range(0, B, mini_size):
                mini_rows = list(range(m0, min(B, m0 + mini_size)))
                local_tok = float(mask_grid[mini_rows].sum())
                # the ranks of a CP group hold the same rows: count them once
                global_tok = max(all_reduce_sum(local_tok, self.state) / self.cp, 1.0)
                micro = make_micro_batches([lens[r] for r in mini_rows], rows_per_micro=rows_per_micro,
                                           token_budget=token_budget)
                t0 = time.perf_counter()
                for mb in micro:
                    rows = [mini_rows[i] for i in mb]
                    stats = self._micro_step(batch, rows, mask_grid, algo_cfg, algorithm, global_tok, temperature,
                                             lens_h)
                    for k in sums:
                        sums[k] += stats.get(k, 0.0)
                t_fwd_bwd += time.perf_counter() - t0
                lr = self.sched.current if self.sched else None
                opt_stats = self.opt.step(lr)
                if self.model.fp8_training is not None:
                    self.model.fp8_training.weights_updated()   # quantised weights are stale now
                for k in opt_t:
                    opt_t[k] += self.opt.last_timing.get(k, 0.0)
                if self.sched:
                    self.sched.step()
        sums = {k: float(v) for k, v in sums.items()}
        tok = max(sums["tok"], 1.0)
        metrics.update({
            "actor/pg_loss": sums["pg_loss"], "actor/ppo_kl": sums["ppo_kl"] / tok,
            "actor/pg_clipfrac": sums["clipfrac"] / tok, "actor/grad_norm": opt_stats.get("grad_norm", 0.0),
            "actor/lr": opt_stats.get("lr", 0.0), "actor/update_skipped": opt_stats.get("skipped", 0.0),
            "timing/fwd_bwd_s": t_fwd_bwd,
            "timing/opt_rs_s": opt_t["opt_rs_s"], "timing/opt_bcast_s": opt_t["opt_bcast_s"],
        })
        if rstats is not None:
            metrics.update(rstats.summary("moe/"))   # router entropy and expert load of this update
        return metrics

    def plan_recompute(self, tokens_per_micro: int, margin_bytes: int = 8 << 30) -> int:
        """Recompute as few decoder layers as the free memory allows: keep the
        activations of as many layers as fit into what is free after the
        resident state (weights, fp32 grads, optimizer shards), less a margin
        for the LM-head chunks, GEMM workspaces and fragmentation."""
        free, _ = torch.cuda.mem_get_info(self.device)
        free += torch.cuda.memory_reserved(self.device) - torch.cuda.memory_allocated(self.device)
        per_layer = int(self.model.activation_bytes_per_token_layer() * tokens_per_micro * 1.1)
        L = self.args.num_layers
        keep = max(0, min(L, (free - margin_bytes) // max(per_layer, 1)))
        n = L - keep
        self.model.recompute_layers = set(range(n))
        return n

    def _micro_step(self, batch: DataProto, rows: list[int], mask_grid: Tensor, algo_cfg, algorithm: str,
                    global_tok: float, temperature: float, lens_h=None) -> dict:
        t = batch.tensors
        pl, rl = lens_h if lens_h is not None else (t["prompt_lengths"], t["response_lengths"])
        pb = pack_from_grid(t["prompt_ids"], pl, t["responses"], rl, rows, self.device, self.cp, self.cp_rank)
        self._set_replay(batch, pb)
        logp, _ = self._forward_scored(pb, temperature, want_entropy=False)
        r_idx = torch.as_tensor(rows, device=self.device)[pb.out_row]
        c_idx = pb.out_col
        old = t["old_log_probs"][r_idx, c_idx].float()
        adv = t["advantages"]
        adv = adv[r_idx] if adv.dim() == 1 else adv[r_idx, c_idx]
        mask = mask_grid[r_idx, c_idx]
        isw = t["rollout_is_weights"][r_idx, c_idx].float() if "rollout_is_weights" in t else None
        if algorithm == "dapo":
            lo, hi, c = float(algo_cfg.clip_ratio_low), float(algo_cfg.clip_ratio_high), float(algo_cfg.clip_ratio_c)
        else:
            lo = hi = float(getattr(algo_cfg, "clip_ratio", 0.2))
            c, isw = 0.0, (isw if algorithm == "grpo_tis" else None)
        loss = ops.ppo_clip_loss(logp, old, adv.float(), mask, lo, hi, c, isw, denom=global_tok)
        kl_c = float(getattr(algo_cfg, "kl_coeff", 0.0))
        if kl_c > 0 and "ref_log_probs" in t:
            ref_lp = t["ref_log_probs"][r_idx, c_idx].float()
            loss = loss + kl_c * ((ref_lp - logp) * mask).sum() / global_tok
        for aux in self.model.aux_losses:
            loss = loss + aux * (mask.sum() / global_tok)
        loss.backward()
        self.model.routing_replay = None
        with torch.no_grad():
            d = logp.detach() - old
            ratio = torch.exp(d.clamp(-20, 20))
            clipped = ((ratio < 1 - lo) | (ratio > 1 + hi)).float()
            return {"pg_loss": loss.detach(), "ppo_kl": ((-d) * mask).sum(), "clipfrac": (clipped * mask).sum(),
                    "tok": mask.sum()}

    # ------------------------------------------------------------------ state
    def state_dict(self) -> dict[str, Any]:
        sd: dict[str, Any] = {"args": self.args.to_dict()}
        if self.opt is not None:
            sd["optimizer"] = self.opt.state_dict()
        if self.sched is not None:
            sd["scheduler"] = self.sched.state_dict()
        return sd
