"""Worker roles hosted by ``WorkerGroup`` processes (one per GPU).

Role contracts follow the reference ABCs (``lumenrl/architecture/abc/
worker_roles.py:10-62``): ``init_model``, ``compute_log_probs``,
``update_policy``, ``get_state_dict``, ``generate``, ``update_weights``,
``compute_rewards``, ``compute_values``, ``compute_teacher_outputs``.  Each
role is a thin shell over the engines, so the same code runs under the
multi-process controller and inside a single torchrun process.
"""

from __future__ import annotations

import os
import socket
from typing import Any, Optional

import torch

from lumenrl_b200.core.config import LumenRLConfig
from lumenrl_b200.core.protocol import DataProto
from lumenrl_b200.core.registry import WORKER_REGISTRY


class BaseWorker:
    """Pins the GPU chosen by the controller before CUDA initialises, and joins
    the process group on request."""

    def __init__(self, config: Optional[dict] = None, **_: Any) -> None:
        gpu = os.environ.get("LUMENRL_WORKER_GPU")
        if gpu is not None and "CUDA_VISIBLE_DEVICES_LOCKED" not in os.environ:
            os.environ["CUDA_VISIBLE_DEVICES"] = str(gpu)
            os.environ["LOCAL_RANK"] = "0"
        self.config = LumenRLConfig.from_dict(config) if isinstance(config, dict) else (config or LumenRLConfig())
        self.rank = int(os.environ.get("RANK", "0"))
        self.world_size = int(os.environ.get("WORLD_SIZE", "1"))
        self.state = None

    def setup_distributed(self, backend: Optional[str] = None, timeout_s: float = 600.0):
        from lumenrl_b200.parallel.dist import init_distributed
        self.state = init_distributed(backend=backend, timeout_s=timeout_s)
        return {"rank": self.state.rank, "world_size": self.state.world_size}

    def get_node_ip(self) -> str:
        return socket.gethostbyname(socket.gethostname()) if socket.gethostname() else "127.0.0.1"

    def get_free_port(self) -> int:
        from lumenrl_b200.controller.worker_group import free_port
        return free_port()

    def get_colocation_info(self) -> dict:
        return {"rank": self.rank, "gpu": os.environ.get("CUDA_VISIBLE_DEVICES"), "pid": os.getpid()}

    def ping(self) -> str:
        return "pong"

    def _ps(self):
        from lumenrl_b200.parallel.dist import ParallelState, get_state
        if self.state is None:
            self.state = get_state() if get_state().world_size > 1 else ParallelState(
                device=torch.device("cuda", 0) if torch.cuda.is_available() else torch.device("cpu"))
        return self.state


def _model_args(config: LumenRLConfig, override=None):
    from lumenrl_b200.models.config import ModelArgs, resolve_model
    if isinstance(override, ModelArgs):
        return override
    if isinstance(override, dict):
        return ModelArgs(**override)
    return resolve_model(config.policy.model_name or "tiny-llama")


class ActorWorker(BaseWorker):
    """Policy: log-probs, policy updates, weights export and checkpoints."""

    def init_model(self, model_args=None, trainable: bool = True) -> dict:
        from lumenrl_b200.engine.training.actor import ActorEngine
        p = self.config.policy
        self.engine = ActorEngine(_model_args(self.config, model_args), self._ps(), lr=p.learning_rate,
                                  betas=(p.adam_beta1, p.adam_beta2), eps=p.adam_eps, weight_decay=p.weight_decay,
                                  max_grad_norm=p.max_grad_norm, seed=self.config.seed, trainable=trainable,
                                  total_steps=self.config.num_training_steps, warmup_steps=p.lr_warmup_steps,
                                  lr_style=p.lr_decay_style)
        return {"num_params": self.engine.args.num_params()}

    def compute_log_probs(self, data: DataProto, temperature: float = 1.0) -> DataProto:
        d = data.to(self.engine.device)
        lp, ent = self.engine.compute_log_probs(d, temperature)
        return DataProto({"old_log_probs": lp, "entropy": ent})

    def update_policy(self, data: DataProto) -> dict:
        algo = self.config.algorithm.name.lower()
        acfg = getattr(self.config.algorithm, algo)
        d = data.to(self.engine.device)
        return self.engine.update_policy(d, acfg, algo, rows_per_micro=self.config.policy.train_micro_batch_size,
                                         num_mini_batches=int(getattr(acfg, "num_mini_batches", 1)),
                                         num_epochs=int(getattr(acfg, "num_ppo_epochs", 1)))

    train_step = update_policy

    def get_flat_weights(self) -> torch.Tensor:
        return self.engine.model.flat.detach().cpu()

    def get_state_dict(self) -> dict:
        return {k: v.detach().cpu().clone() for k, v in self.engine.model.hf_state_dict().items()}

    def export_state_dict_safetensors(self, out_dir: str) -> list[str]:
        from lumenrl_b200.utils.checkpoint import save_hf_safetensors
        return save_hf_safetensors(self.engine.model, out_dir) if self.rank == 0 else []

    def save_checkpoint(self, path: str, step: int) -> str:
        from lumenrl_b200.utils.checkpoint import save_sharded
        return save_sharded(self.engine, path, step, self.rank, self.world_size)

    def load_checkpoint(self, path: str) -> int:
        from lumenrl_b200.utils.checkpoint import load_sharded
        return load_sharded(self.engine, path, self.rank, self.world_size)


class RefWorker(ActorWorker):
    def init_model(self, model_args=None, trainable: bool = False) -> dict:
        return super().init_model(model_args, trainable=False)

    def compute_ref_log_probs(self, data: DataProto, temperature: float = 1.0) -> DataProto:
        out = self.compute_log_probs(data, temperature)
        return DataProto({"ref_log_probs": out["old_log_probs"]})

    def load_weights(self, flat: torch.Tensor) -> None:
        self.engine.model.flat.copy_(flat.to(self.engine.model.flat.device))


class RolloutWorker(BaseWorker):
    """Native engine on its own copy of the weights (separated mode) or on
    the actor's buffer (hybrid/colocated)."""

    def init_model(self, model_args=None, max_num_seqs: int = 64, max_model_len: int = 2048) -> dict:
        from lumenrl_b200.engine.inference.engine import RolloutEngine
        from lumenrl_b200.models.qwen3 import Qwen3Model
        st = self._ps()
        args = _model_args(self.config, model_args)
        dtype = torch.bfloat16 if st.device.type == "cuda" else torch.float32
        self.model = Qwen3Model(args, device=st.device, dtype=dtype, requires_grad=False)
        self.model.init_weights(self.config.seed)
        vc = self.config.policy.generation.vllm_cfg
        self.engine = RolloutEngine(self.model, max_num_seqs=max_num_seqs, max_model_len=max_model_len,
                                    use_cuda_graph=not vc.enforce_eager or st.device.type == "cuda")
        self.temperature, self.top_p = float(vc.temperature), float(vc.top_p)
        return {"kv_blocks": self.engine.cache.num_blocks}

    def generate(self, data: DataProto, n: int = 1, max_new_tokens: int = 128, seed: int = 0,
                 eos_token_id: Optional[int] = None) -> DataProto:
        from lumenrl_b200.engine.inference.engine import SamplingParams
        prompts = data["prompt_ids"].to(self.engine.device)
        out = self.engine.generate(prompts, SamplingParams(max_new_tokens=max_new_tokens, temperature=self.temperature,
                                                           top_p=self.top_p, n=n, seed=seed + self.rank,
                                                           eos_token_id=eos_token_id))
        d = DataProto({"prompt_ids": out.prompts, "responses": out.responses,
                       "response_lengths": out.response_lengths, "rollout_log_probs": out.logprobs})
        if out.routed_experts:
            d.ragged["routed_experts"] = out.routed_experts
        return d

    def update_weights(self, flat: torch.Tensor, version: Optional[int] = None) -> int:
        self.engine.update_weights(flat.to(self.engine.device), version)
        return self.engine.weight_version

    def update_weights_from_path(self, path: str) -> int:
        from lumenrl_b200.utils.checkpoint import load_hf_safetensors
        load_hf_safetensors(self.model, path)
        self.engine.update_weights()
        return self.engine.weight_version

    def sleep(self) -> None:
        self.engine.sleep()

    def wake(self) -> None:
        self.engine.wake()


class RewardWorker(BaseWorker):
    def init_model(self, reward: Optional[str] = None, **kw) -> None:
        from lumenrl_b200.rewards import get_reward_fn
        self.fn = get_reward_fn(reward or self.config.reward.function)
        self.kw = kw

    def compute_rewards(self, data: DataProto) -> DataProto:
        r = self.fn(data["responses"], None, lengths=data.tensors.get("response_lengths"), **self.kw)
        return DataProto({"rewards": r.float().cpu()})


class CriticWorker(BaseWorker):
    """Value model: the policy architecture with a scalar head per token."""

    def init_model(self, model_args=None) -> dict:
        from lumenrl_b200.engine.training.critic import CriticEngine
        c = self.config.critic
        self.engine = CriticEngine(_model_args(self.config, model_args), self._ps(), lr=c.learning_rate,
                                   weight_decay=c.weight_decay, max_grad_norm=c.max_grad_norm, seed=self.config.seed)
        return {"num_params": self.engine.args.num_params()}

    def compute_values(self, data: DataProto) -> DataProto:
        return DataProto({"values": self.engine.compute_values(data.to(self.engine.device))})

    def update_critic(self, data: DataProto) -> dict:
        return self.engine.update(data.to(self.engine.device), self.config.critic.value_clip_ratio,
                                  self.config.policy.train_micro_batch_size)

    train_step = update_critic


class TeacherWorker(BaseWorker):
    """Frozen teacher: logits or auxiliary hidden states (Eagle3 / OPD)."""

    def init_model(self, model_args=None, aux_layers: Optional[list[int]] = None) -> dict:
        from lumenrl_b200.models.qwen3 import Qwen3Model
        st = self._ps()
        args = _model_args(self.config, model_args)
        dtype = torch.bfloat16 if st.device.type == "cuda" else torch.float32
        self.model = Qwen3Model(args, device=st.device, dtype=dtype, requires_grad=False)
        self.model.init_weights(self.config.seed)
        self.aux_layers = aux_layers or []
        return {"layers": args.num_layers}

    @torch.no_grad()
    def compute_teacher_outputs(self, data: DataProto, want_logits: bool = False) -> DataProto:
        ids = data["input_ids"].to(self.model.flat.device)
        cu = data["cu_seqlens"].to(self.model.flat.device)
        pos = data["position_ids"].to(self.model.flat.device)
        h, taps = self.model.forward_packed(ids, pos, cu, int((cu[1:] - cu[:-1]).max()),
                                            output_hidden_layers=self.aux_layers)
        out = {"last_hidden_states": h}
        if taps:
            out["aux_hidden_states"] = torch.cat(taps, -1)
        if want_logits:
            out["teacher_logits"] = self.model.logits(h)
        return DataProto(out)


class HybridWorker(ActorWorker):
    """Actor + rollout engine in one process sharing the flat bf16 weights."""

    def init_model(self, model_args=None, trainable: bool = True, max_num_seqs: int = 64,
                   max_model_len: int = 2048) -> dict:
        info = super().init_model(model_args, trainable)
        from lumenrl_b200.engine.inference.engine import RolloutEngine
        self.rollout = RolloutEngine(self.engine.model, max_num_seqs=max_num_seqs, max_model_len=max_model_len)
        return info

    def generate(self, data: DataProto, **kw) -> DataProto:
        rw = RolloutWorker.__new__(RolloutWorker)
        rw.engine, rw.rank = self.rollout, self.rank
        vc = self.config.policy.generation.vllm_cfg
        rw.temperature, rw.top_p = float(vc.temperature), float(vc.top_p)
        return RolloutWorker.generate(rw, data, **kw)

    def sync_weights(self) -> int:
        self.rollout.update_weights()
        return self.rollout.weight_version


for _k, _v in {"actor": ActorWorker, "ref": RefWorker, "rollout": RolloutWorker, "reward": RewardWorker,
               "critic": CriticWorker, "teacher": TeacherWorker, "hybrid": HybridWorker}.items():
    WORKER_REGISTRY.register(_k, _v)
