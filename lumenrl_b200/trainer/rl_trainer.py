"""Synchronous RL trainer (GRPO / DAPO / PPO), colocated or separated.

Per step (reference hot loop ``lumenrl/trainer/rl_trainer.py:3003-3522``):

1. rollout: every rank generates ``prompts_per_rank x n`` samples with the
   native engine on the policy's own bf16 weights (data-parallel rollout,
   groups never straddle ranks, so advantages need no communication);
2. rewards (programmatic function, or reward model);
3. DAPO dynamic sampling with refill rounds (``filter_groups.enable``): groups
   whose rewards are all equal are dropped and fresh prompts are generated
   until the step has its full count of informative groups or
   ``max_num_gen_batches`` rounds ran (reference ``rl_trainer.py:2163-2189``);
4. old log-probs (skipped in bypass mode) and, when ``kl_coeff > 0`` or
   ``use_kl_in_reward``, reference log-probs from a frozen copy; with
   ``use_kl_in_reward`` the rewards become token-level ``r - beta * KL`` under
   a fixed / adaptive KL controller (reference ``rl_trainer.py:3183``);
5. critic values for GAE when the algorithm is PPO (reference
   ``rl_trainer.py:3189-3193``), then advantages (estimator registry) and
   rollout correction (TIS/MIS/RS);
6. policy update (sharded AdamW), whose final all-gather leaves every GPU with
   the new bf16 weights: that is the weight sync in colocated mode; PPO then
   updates the critic on the same batch (clipped value loss);
7. metrics with the reference's names (``timing/*``, ``perf/throughput``,
   ``rollout_corr/*``, ``actor/*``).

Every phase is timed on the device (CUDA events) when running on GPU.
"""

from __future__ import annotations

import logging
import math
import time
from dataclasses import dataclass, field
from typing import Any, Callable, Optional

import torch

from lumenrl_b200.algorithms import rollout_correction as rc
from lumenrl_b200.core.config import LumenRLConfig
from lumenrl_b200.core.protocol import DataProto
from lumenrl_b200.core.registry import ALGORITHM_REGISTRY
from lumenrl_b200.data.synthetic import SyntheticPrompts
from lumenrl_b200.engine.inference.engine import RolloutEngine, SamplingParams
from lumenrl_b200.engine.training.actor import ActorEngine
from lumenrl_b200.models.config import ModelArgs, resolve_model
from lumenrl_b200.parallel.dist import (ParallelState, all_reduce_max_many, all_reduce_sum_many, get_state,
                                        init_distributed)
from lumenrl_b200.rewards import get_reward_fn
from lumenrl_b200.utils.timers import PhaseTimer

logger = logging.getLogger(__name__)


@dataclass
class RLRunSpec:
    """Workload knobs that the YAML schema does not carry (synthetic runs)."""
    prompts_per_step: int = 8            # global prompts per step
    prompt_len: int = 32
    prompt_low: int = 3
    prompt_high: int = 2048
    max_new_tokens: int = 32
    eos_token_id: Optional[int] = 2
    reward: str = "contains_token"
    reward_kwargs: dict = field(default_factory=dict)
    rows_per_micro: int = 4
    logprob_token_budget: int = 16384
    kv_cache_bytes: Optional[int] = None
    use_cuda_graph: bool = True
    gradient_checkpointing: object = False   # True (every layer), False, or "auto" (memory-budgeted)


def _keep_groups(out, n: int, T: int, member: int):
    """Rows of every T-th prompt group (starting at ``member``) of a
    generation result: whole GRPO groups, so group statistics stay local."""
    from dataclasses import replace
    P = out.responses.shape[0] // n
    keep_p = torch.arange(member, P, T, device=out.responses.device)
    rows = (keep_p.unsqueeze(1) * n + torch.arange(n, device=keep_p.device)).reshape(-1)
    prompts = out.prompts[rows] if isinstance(out.prompts, torch.Tensor) else [out.prompts[i] for i in rows.tolist()]
    return replace(out, prompts=prompts, responses=out.responses[rows], response_lengths=out.response_lengths[rows],
                   logprobs=out.logprobs[rows], prompt_index=out.prompt_index[rows],
                   routed_experts=[out.routed_experts[i] for i in rows.tolist()] if out.routed_experts else [])


class RLTrainer:
    def __init__(self, config: LumenRLConfig, model_args: Optional[ModelArgs] = None,
                 spec: Optional[RLRunSpec] = None, state: Optional[ParallelState] = None) -> None:
        self.config = config
        from lumenrl_b200.ops.kernel_flags import apply_kernels_config
        apply_kernels_config(getattr(config, "kernels", None))   # config's kernel choices win over LRL_*
        self.spec = spec or RLRunSpec()
        self.model_args = model_args or resolve_model(config.policy.model_name or "tiny-llama")
        self.state = state
        self.callbacks: list = []
        self.global_step = 0
        self.history: list[dict] = []

    # ------------------------------------------------------------------ setup
    def setup(self) -> "RLTrainer":
        c = self.config
        if self.state is None:
            self.state = get_state() if get_state().world_size > 1 or get_state().device.type == "cuda" \
                else init_distributed()
        self._setup_training()
        self._setup_rollout(self.actor.model, self.state.world_size)
        return self

    def _setup_training(self) -> None:
        """Algorithm, actor (+ FP8 training, reference, critic), data and
        rewards on ``self.state`` (the trainer's data-parallel group)."""
        c = self.config
        st = self.state
        algo = c.algorithm.name.lower()
        self.algorithm_name = algo
        self.algorithm = ALGORITHM_REGISTRY.get(algo)(c)
        self.algo_cfg = getattr(c.algorithm, algo)
        self.group = int(getattr(self.algo_cfg, "num_generations", 1) or 1)
        p = c.policy
        engine_cls = ActorEngine
        if self._shard_params():
            from lumenrl_b200.engine.training.fsdp import ShardedParamActorEngine
            engine_cls = ShardedParamActorEngine
        self.actor = engine_cls(
            self.model_args, st, lr=p.learning_rate, betas=(p.adam_beta1, p.adam_beta2), eps=p.adam_eps,
            weight_decay=p.weight_decay, max_grad_norm=p.max_grad_norm, seed=c.seed,
            gradient_checkpointing=self.spec.gradient_checkpointing, total_steps=c.num_training_steps,
            warmup_steps=p.lr_warmup_steps, lr_style=p.lr_decay_style,
            min_lr_ratio=(p.min_lr / p.learning_rate if p.learning_rate else 0.0))
        self.fp8_training = None
        if c.quantization.training.fp8:
            # hybrid FP8 training: E4M3 forward, E5M2 gradients, bf16/fp32 master
            from lumenrl_b200.quant.fp8 import FP8Config, FP8TrainingManager
            self.fp8_training = FP8TrainingManager(FP8Config.from_config(c.quantization))
            self.fp8_training.attach(self.actor.model)
        self.ref = None
        kl_coeff = float(getattr(self.algo_cfg, "kl_coeff", 0.0))
        self.kl_ctrl = None
        if c.algorithm.use_kl_in_reward:
            from lumenrl_b200.algorithms.kl_controller import get_kl_controller
            self.kl_ctrl = get_kl_controller(c.algorithm.kl_ctrl_type, kl_coeff, c.algorithm.kl_target,
                                             c.algorithm.kl_horizon)
        if kl_coeff > 0 or self.kl_ctrl is not None:
            self.ref = ActorEngine(self.model_args, st, seed=c.seed, trainable=False, init=False)
            self.ref.model.flat.copy_(self._actor_flat(self.ref.model.flat.numel()))
        self.critic = None
        if algo == "ppo" or c.algorithm.adv_estimator == "gae" or c.critic.enabled:
            from lumenrl_b200.engine.training.critic import CriticEngine
            cc = c.critic
            self.critic = CriticEngine(self.model_args, st, lr=cc.learning_rate, weight_decay=cc.weight_decay,
                                       max_grad_norm=cc.max_grad_norm, seed=c.seed + 1,
                                       gradient_checkpointing=self.spec.gradient_checkpointing,
                                       total_steps=c.num_training_steps)
        self._setup_common()

    def _shard_params(self) -> bool:
        """Colocated: the trainer's resident weights are the rollout engine's,
        so they are never sharded (see ``ShardedParamActorEngine``)."""
        return False

    def _actor_flat(self, numel: Optional[int] = None) -> torch.Tensor:
        """The actor's whole bf16 model as one flat buffer (assembled from the
        shards when the weights are sharded)."""
        if self.actor.model.flat is not None:
            return self.actor.model.flat
        return self.actor.full_flat(numel)

    def _setup_common(self) -> None:
        c, st = self.config, self.state
        if not hasattr(self, "algorithm_name"):
            self.algorithm_name = c.algorithm.name.lower()
            self.algo_cfg = getattr(c.algorithm, self.algorithm_name)
            self.group = int(getattr(self.algo_cfg, "num_generations", 1) or 1)
        vc = c.policy.generation.vllm_cfg
        self.temperature = float(vc.temperature)
        self.top_p = float(vc.top_p)
        self.data = SyntheticPrompts(self.spec.prompt_len, self.spec.prompt_low, self.spec.prompt_high, c.seed)
        self.reward_fn = get_reward_fn(self.spec.reward)
        from lumenrl_b200.utils.profiler import DistProfiler
        self.profiler = DistProfiler(c.profiler, st.rank)
        # NVTX ranges per phase whenever profiling is on for this rank
        self.timer = PhaseTimer(st.device, nvtx=self.profiler.enabled)
        self.io_bytes = {"h2d": 0, "d2h": 0}

    def _setup_rollout(self, model, rollout_ranks: int) -> None:
        """Rollout engine over ``model`` (the trainer's own weights when
        colocated); ``rollout_ranks`` split the step's prompts."""
        c = self.config
        vc = c.policy.generation.vllm_cfg
        max_len = self.spec.prompt_len + self.spec.max_new_tokens
        prompts_per_rank = max(1, self.spec.prompts_per_step // rollout_ranks)
        self.prompts_per_rank = prompts_per_rank
        # rollout tensor parallelism: TP groups of consecutive ranks generate
        # the same prompts together; each member then keeps every T-th GRPO
        # group of the result, so training stays data parallel over all ranks
        T = int(getattr(vc, "tensor_parallel_size", 1) or 1)
        self.tp_size, self.tp_member, self.tp_group = T, 0, None
        if T > 1:
            import torch.distributed as dist
            W, r = self.state.world_size, self.state.rank
            if W % T:
                raise ValueError(f"rollout tensor_parallel_size={T} must divide the {W} rollout ranks")
            groups = [dist.new_group(list(range(g * T, (g + 1) * T))) for g in range(W // T)]  # every rank, same order
            self.tp_group, self.tp_member = groups[r // T], r % T
        kv_dtype = torch.float8_e4m3fn if str(vc.kv_cache_dtype).startswith("fp8") else torch.bfloat16
        self.rollout = RolloutEngine(model, max_num_seqs=prompts_per_rank * T * self.group,
                                     max_model_len=max_len, kv_cache_bytes=self.spec.kv_cache_bytes,
                                     use_cuda_graph=self.spec.use_cuda_graph, kv_dtype=kv_dtype,
                                     fp8_rollout=self._fp8_rollout_config(c), tp_group=self.tp_group)

    @staticmethod
    def _fp8_rollout_config(c):
        """quantization.rollout.precision = fp8 -> blockwise W8A8 rollout."""
        from lumenrl_b200.quant.fp8 import FP8Config
        r = c.quantization.rollout
        if "fp8" not in str(getattr(r, "precision", "bf16")).lower():
            return None
        return FP8Config(precision=r.precision, num_first_layers_in_bf16=r.num_first_layers_in_bf16,
                         num_last_layers_in_bf16=r.num_last_layers_in_bf16)

    # ------------------------------------------------------------------ step
    def _rollout(self, step: int, round_idx: int = 0) -> DataProto:
        st, sp = self.state, self.spec
        T = getattr(self, "tp_size", 1)
        src = st.rank // T          # the members of a rollout TP group draw the same prompts and samples
        host = self.data.batch_tensor(self.prompts_per_rank * T, step, src, pin=st.device.type == "cuda",
                                      round=round_idx)
        prompts = host.to(st.device, non_blocking=True)
        self.io_bytes["h2d"] = host.numel() * host.element_size()
        params = SamplingParams(max_new_tokens=sp.max_new_tokens, temperature=self.temperature, top_p=self.top_p,
                                n=self.group,
                                seed=self.config.seed * 7919 + step * 131 + src + round_idx * 1_000_033,
                                eos_token_id=sp.eos_token_id)
        self.rollout.wake()
        out = self.rollout.generate(prompts, params)
        self.rollout.sleep()
        if T > 1:
            out = _keep_groups(out, self.group, T, self.tp_member)
        dev = st.device
        B = out.responses.shape[0]
        pgrid = out.prompts
        plens = torch.full((B,), pgrid.shape[1], dtype=torch.long, device=dev)
        R = out.responses.shape[1]
        rmask = (torch.arange(R, device=dev).unsqueeze(0) < out.response_lengths.unsqueeze(1)).float()
        batch = DataProto(
            tensors={"prompt_ids": pgrid, "prompt_lengths": plens, "responses": out.responses,
                     "response_lengths": out.response_lengths, "response_mask": rmask,
                     "rollout_log_probs": out.logprobs},
            meta={"num_generations": self.group,
                  "uid": [f"{step}-{st.rank}-{round_idx}-{int(i)}" for i in out.prompt_index.tolist()],
                  "response_lengths": out.response_lengths.tolist(), "gen_stats": out.stats})
        if out.routed_experts:
            batch.ragged["routed_experts"] = out.routed_experts
        return batch

    def _tp_total(self, n: int) -> int:
        """``n`` summed over this rank's rollout TP group (a generation round is
        collective inside the group, so its members decide refills together)."""
        if getattr(self, "tp_size", 1) <= 1:
            return n
        import torch.distributed as dist
        t = torch.tensor([float(n)], device=self.state.device)
        dist.all_reduce(t, group=self.tp_group)
        return int(t.item())

    def _score(self, batch: DataProto) -> None:
        rewards = self.reward_fn(batch["responses"], None, lengths=batch["response_lengths"], **self.spec.reward_kwargs)
        batch["rewards"] = rewards.to(self.state.device).float()

    def _collect(self, step: int, m: dict) -> DataProto:
        """One rollout round, or DAPO refill rounds until ``prompts_per_rank``
        groups with non-constant rewards are collected."""
        c = self.config
        fg = c.algorithm.dapo.filter_groups
        if not (self.algorithm_name == "dapo" and fg.enable):
            batch = self._rollout(step)
            self._score(batch)
            return batch
        from lumenrl_b200.algorithms.dapo_sampling import filter_groups_keep_mask
        max_rounds = int(fg.max_num_gen_batches) if int(fg.max_num_gen_batches) > 0 else 10_000
        parts, uids, stats, kept, rounds, seen = [], [], {}, 0, 0, 0
        while self._tp_total(kept) < self.prompts_per_rank * getattr(self, "tp_size", 1) and rounds < max_rounds:
            b = self._rollout(step, rounds)
            self._score(b)
            keep, kept_uids = filter_groups_keep_mask(b["rewards"].float().cpu(), b.meta["uid"])
            rounds += 1
            seen += len(set(b.meta["uid"]))
            for k, v in b.meta.get("gen_stats", {}).items():
                if isinstance(v, (int, float)):
                    stats[k] = stats.get(k, 0.0) + v
            if bool(keep.any()):
                idx = keep.nonzero(as_tuple=True)[0]
                parts.append(b.select_idxs(idx))
                uids.extend(b.meta["uid"][i] for i in idx.tolist())
                kept += len(kept_uids)
        if not parts:
            raise RuntimeError("DAPO filter_groups kept no prompt group in "
                               f"{rounds} generation round(s); raise max_num_gen_batches or check the reward")
        batch = DataProto.merge(parts)
        n_rows = min(len(batch), self.prompts_per_rank * self.group)
        if n_rows < len(batch):
            batch = batch.select_idxs(torch.arange(n_rows))
            uids = uids[:n_rows]
        batch.meta.update({"num_generations": self.group, "uid": uids,
                           "response_lengths": batch["response_lengths"].tolist(), "gen_stats": stats})
        m["dapo/gen_rounds"] = float(rounds)
        m["dapo/kept_groups"] = float(len(uids) // self.group)
        m["dapo/kept_frac"] = kept / max(seen, 1)
        return batch

    def step(self) -> dict[str, Any]:
        c, st = self.config, self.state
        step = self.global_step
        m: dict[str, Any] = {}
        self.profiler.start(step)               # no-op unless profiling this rank and step
        self.timer.start("step")
        self.timer.start("gen")
        batch = self._collect(step, m)
        self.timer.stop("gen")
        scores = batch["rewards"]
        if self.algorithm_name == "dapo" and c.algorithm.dapo.filter_groups.enable and "dapo/kept_frac" not in m:
            from lumenrl_b200.algorithms.dapo_sampling import filter_groups_keep_mask
            keep, _ = filter_groups_keep_mask(batch["rewards"].cpu(), batch.meta["uid"])
            m["dapo/kept_frac"] = float(keep.float().mean())
        rcfg = c.quantization.rollout_correction
        self.timer.start("old_log_prob")
        if rcfg.bypass_mode:
            rc.apply_bypass_mode(batch, rcfg)
        else:
            lp, ent = self.actor.compute_log_probs(batch, self.temperature, self.spec.logprob_token_budget)
            batch["old_log_probs"] = lp
            mask = batch["response_mask"]
            m["actor/entropy"] = float((ent * mask).sum() / mask.sum().clamp(min=1))
        self.timer.stop("old_log_prob")
        if self.ref is not None:
            self.timer.start("ref")
            batch["ref_log_probs"], _ = self.ref.compute_log_probs(batch, self.temperature,
                                                                   self.spec.logprob_token_budget, want_entropy=False)
            self.timer.stop("ref")
        if self.kl_ctrl is not None:
            from lumenrl_b200.algorithms.kl_controller import apply_kl_penalty
            batch, klm = apply_kl_penalty(batch, self.kl_ctrl, c.algorithm.kl_penalty)
            m.update(klm)
            del batch.tensors["ref_log_probs"]     # the KL is in the reward, not in the policy loss
        if self.critic is not None:
            self.timer.start("values")
            batch["values"] = self.critic.compute_values(batch, self.spec.logprob_token_budget)
            self.timer.stop("values")
        self.timer.start("adv")
        self.algorithm.compute_advantages(batch)
        if rcfg.rollout_is or rcfg.rollout_rs:
            batch, corr = rc.compute_rollout_correction_and_add_to_batch(batch, rcfg)
            m.update(corr)
        else:
            m.update(rc.compute_rollout_corr_metrics_from_logprobs(batch["old_log_probs"], batch["rollout_log_probs"],
                                                                   batch["response_mask"]))
        mm = rc.mismatch_sums(batch["old_log_probs"], batch["rollout_log_probs"], batch["response_mask"]) \
            if "old_log_probs" in batch.tensors and "rollout_log_probs" in batch.tensors else None
        self.timer.stop("adv")
        self.timer.start("train")
        pol = c.algorithm.dapo if self.algorithm_name == "dapo" else self.algo_cfg
        tm = self.actor.update_policy(batch, pol, self.algorithm_name, rows_per_micro=self.spec.rows_per_micro,
                                      num_mini_batches=int(getattr(self.algo_cfg, "num_mini_batches", 1)),
                                      num_epochs=int(getattr(self.algo_cfg, "num_ppo_epochs", 1)),
                                      temperature=self.temperature)
        self.timer.stop("train")
        if self.critic is not None:
            self.timer.start("critic")
            for _ in range(max(1, int(c.critic.num_critic_epochs))):
                tm.update(self.critic.update(batch, clip=float(c.critic.value_clip_ratio),
                                             rows_per_micro=self.spec.rows_per_micro))
            self.timer.stop("critic")
        self.timer.start("weight_sync")
        m.update(self._sync_weights())
        self.timer.stop("weight_sync")
        self.timer.stop("step")
        times = self.timer.collect()
        m.update(tm)
        # every cross-rank statistic of the step in two collectives (one sum
        # vector, one max vector) and two device->host reads
        resp_local = batch["response_lengths"].sum()
        local = torch.stack([batch["prompt_lengths"].sum() + resp_local, resp_local, scores.sum()]).double()
        if mm is not None:
            local = torch.cat([local, mm.to(local.device)])
        local = local.cpu().tolist()
        summed = all_reduce_sum_many(local[:3] + [float(len(batch))] + local[3:])
        tokens, resp_tokens, score_sum, rows = summed[:4]
        if mm is not None:
            m.update(rc.finalize_mismatch(summed[4:]))
        # Weight sync = from the reduced gradients to rollout-ready weights: the
        # AdamW kernel that writes bf16 into the resident buffer the engine
        # reads (and, on several GPUs, stores it into every rank's copy over
        # NVLink), plus the engine-side update (fp8 re-quantisation when the
        # rollout runs W8A8; a pointer check otherwise).  Max over ranks.
        opt_keys = [k for k in ("timing/opt_rs_s", "timing/opt_bcast_s") if k in m]
        max_keys = [f"timing/{k}_s" for k in times] + opt_keys + ["timing/weight_sync_s"]
        max_vals = list(times.values()) + [float(m[k]) for k in opt_keys] + [
            float(tm.get("timing/opt_bcast_s", 0.0)) + times["weight_sync"]]
        if st.device.type == "cuda":    # memory high-water marks of this step's process, max over ranks
            gb = float(1 << 30)
            max_keys += ["mem/actor_max_reserved_gb", "mem/actor_max_allocated_gb", "mem/actor_reserved_gb",
                         "mem/actor_allocated_gb"]
            max_vals += [torch.cuda.max_memory_reserved(st.device) / gb, torch.cuda.max_memory_allocated(st.device) / gb,
                         torch.cuda.memory_reserved(st.device) / gb, torch.cuda.memory_allocated(st.device) / gb]
        m.update(zip(max_keys, all_reduce_max_many(max_vals)))
        step_s = m["timing/step_s"]
        m["perf/total_num_tokens"] = tokens
        m["perf/step_tokens_per_s"] = tokens / step_s
        m["perf/throughput"] = tokens / (step_s * st.world_size)
        m["perf/gen_tokens_per_s"] = resp_tokens / max(m["timing/gen_s"], 1e-9)
        m["reward/mean"] = score_sum / rows
        m["response_length/mean"] = resp_tokens / rows
        sync_s = m["timing/weight_sync_s"]
        m["weight_sync/ms"] = sync_s * 1e3
        wbytes = sum(p.numel() for _, p in self.actor.model.named_flat_params()) * (
            2 if self.actor.model.p("embed").dtype == torch.bfloat16 else 4)
        m["weight_sync/GBps"] = wbytes / max(sync_s, 1e-9) / 1e9
        for k in ("prefill_ms", "setup_ms", "decode_ms"):
            if k in batch.meta.get("gen_stats", {}):
                m[f"timing/gen_{k}"] = batch.meta["gen_stats"][k]
        self.last_trace = self.profiler.stop() or getattr(self, "last_trace", None)   # chrome trace path
        host_result = scores.to("cpu")          # the step's result read back to the host
        self.io_bytes["d2h"] = host_result.numel() * host_result.element_size()
        m["step"] = step + 1
        self.global_step += 1
        self.history.append(m)
        for cb in self.callbacks:
            cb.on_step_end(self, m)
        return m

    def _sync_weights(self) -> dict:
        """Colocated: the engine reads the trainer's resident buffer (the
        optimizer kernel already wrote the new weights there); only the FP8
        rollout re-quantises.  Overridden by the separated trainer."""
        self.rollout.update_weights()
        return {}

    def train(self) -> list[dict]:
        for cb in self.callbacks:
            cb.on_train_begin(self)
        for _ in range(self.global_step, self.config.num_training_steps):
            self.step()
        for cb in self.callbacks:
            cb.on_train_end(self)
        return self.history

    def cleanup(self) -> None:
        self.rollout.sleep()
