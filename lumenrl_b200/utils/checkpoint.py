"""Checkpoints: sharded resume state and HF-safetensors export.

Resume layout (one directory per step, 1-based like the reference's
``global_step_N``; reference ``lumenrl/workers/actor_worker.py:1045-1166``,
``lumenrl/trainer/callbacks.py:55-186``)::

    <root>/global_step_<N>/actor/
        model_world_size_<W>_rank_<R>.pt      # this rank's fp32 master shard + Adam m/v + step
        extra_state_world_size_<W>_rank_<R>.pt  # scheduler, RNG states, data cursor
        weights_bf16.safetensors              # (rank 0) full bf16 weights, flat layout
    <root>/latest_checkpointed_iteration.txt

HF export writes ``model-0000x-of-0000y.safetensors`` shards with HF parameter
names plus ``model.safetensors.index.json`` and a ``config.json``, so the
result loads with ``transformers`` (reference ``rl_trainer.py:1592-1635``).
``CheckpointManager`` prunes to ``save_total_limit``.
"""

from __future__ import annotations

import json
import os
import random
import re
import shutil
from typing import Optional

import numpy as np
import torch

TRACKER = "latest_checkpointed_iteration.txt"


def _step_dir(root: str, step: int) -> str:
    return os.path.join(root, f"global_step_{step}", "actor")


def _atomic(path: str, write) -> None:
    """write(tmp_path) then rename into place: a crash leaves either the old
    file or none, never a truncated one."""
    tmp = f"{path}.tmp{os.getpid()}"
    write(tmp)
    os.replace(tmp, path)


def _all_ranks_done(world: int) -> None:
    import torch.distributed as dist
    if world > 1 and dist.is_available() and dist.is_initialized():
        dist.barrier()


def save_sharded(engine, root: str, step: int, rank: int, world: int, extra: Optional[dict] = None) -> str:
    """Every rank writes its shard files (each to a temporary name, renamed
    when complete); after all ranks have written, rank 0 publishes the step
    in the tracker file (also by rename).  A crash at any point leaves the
    tracker naming the previous complete step, mirroring the reference's
    order (tracker only after every rank's save, reference
    ``lumenrl/trainer/callbacks.py:170-178``).  Must be called on every rank."""
    d = _step_dir(root, step)
    os.makedirs(d, exist_ok=True)
    opt = engine.opt
    state = {"optimizer": {k: (v.detach().cpu() if torch.is_tensor(v) else v) for k, v in opt.state_dict().items()},
             "args": engine.args.to_dict()}
    _atomic(os.path.join(d, f"model_world_size_{world}_rank_{rank}.pt"), lambda p: torch.save(state, p))
    ex = {"scheduler": engine.sched.state_dict() if engine.sched else None,
          "rng": {"torch": torch.get_rng_state(), "numpy": np.random.get_state(), "python": random.getstate(),
                  "cuda": torch.cuda.get_rng_state_all() if torch.cuda.is_available() else None},
          **(extra or {})}
    _atomic(os.path.join(d, f"extra_state_world_size_{world}_rank_{rank}.pt"), lambda p: torch.save(ex, p))
    if rank == 0:
        from safetensors.torch import save_file
        flat = {"flat": engine.model.flat.detach().cpu().contiguous()}
        _atomic(os.path.join(d, "weights_bf16.safetensors"), lambda p: save_file(flat, p))
    _all_ranks_done(world)
    if rank == 0:
        def _tracker(p):
            with open(p, "w") as f:
                f.write(str(step))
        _atomic(os.path.join(root, TRACKER), _tracker)
    return d


def latest_step(root: str) -> Optional[int]:
    p = os.path.join(root, TRACKER)
    if os.path.isfile(p):
        with open(p) as f:
            return int(f.read().strip())
    steps = [int(m.group(1)) for n in (os.listdir(root) if os.path.isdir(root) else [])
             if (m := re.fullmatch(r"global_step_(\d+)", n))]
    return max(steps) if steps else None


def load_sharded(engine, root: str, rank: int, world: int, step: Optional[int] = None, data=None) -> int:
    """Restore the optimizer shard, scheduler, host and CUDA RNG streams and,
    when ``data`` (an object with ``load_state_dict``) is given, the data
    cursor saved under the ``data`` key.  Returns the restored step (0 when
    nothing was saved)."""
    step = latest_step(root) if step is None else step
    if step is None:
        return 0
    d = _step_dir(root, step)
    state = torch.load(os.path.join(d, f"model_world_size_{world}_rank_{rank}.pt"), map_location="cpu",
                       weights_only=False)
    engine.opt.load_state_dict({k: (v.to(engine.device) if torch.is_tensor(v) else v)
                                for k, v in state["optimizer"].items()})
    ex = torch.load(os.path.join(d, f"extra_state_world_size_{world}_rank_{rank}.pt"), map_location="cpu",
                    weights_only=False)
    if engine.sched is not None and ex.get("scheduler"):
        engine.sched.load_state_dict(ex["scheduler"])
    rng = ex.get("rng") or {}
    if "torch" in rng:
        torch.set_rng_state(rng["torch"])
    if "numpy" in rng:
        np.random.set_state(rng["numpy"])
    if "python" in rng:
        random.setstate(rng["python"])
    if rng.get("cuda") is not None and torch.cuda.is_available():
        saved = rng["cuda"]
        if len(saved) == torch.cuda.device_count():
            torch.cuda.set_rng_state_all(saved)
        else:   # different device count: restore what this process's device had
            torch.cuda.set_rng_state(saved[min(torch.cuda.current_device(), len(saved) - 1)])
    if data is not None and ex.get("data") is not None:
        data.load_state_dict(ex["data"])
    return step


def save_hf_safetensors(model, out_dir: str, max_shard_bytes: int = 5 * 1024 ** 3,
                        dtype: torch.dtype = torch.bfloat16) -> list[str]:
    """HF-named safetensors shards + index + config.json."""
    from safetensors.torch import save_file
    os.makedirs(out_dir, exist_ok=True)
    sd = model.hf_state_dict()
    shards: list[dict] = [{}]
    size = 0
    for k, v in sd.items():
        nb = v.numel() * torch.empty(0, dtype=dtype).element_size()
        if size + nb > max_shard_bytes and shards[-1]:
            shards.append({})
            size = 0
        shards[-1][k] = v.detach().to(dtype).contiguous().cpu()
        size += nb
    files, index = [], {}
    total = 0
    for i, sh in enumerate(shards):
        name = f"model-{i + 1:05d}-of-{len(shards):05d}.safetensors"
        save_file(sh, os.path.join(out_dir, name), metadata={"format": "pt"})
        files.append(name)
        for k, v in sh.items():
            index[k] = name
            total += v.numel() * v.element_size()
    with open(os.path.join(out_dir, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {"total_size": total}, "weight_map": index}, f, indent=2)
    with open(os.path.join(out_dir, "config.json"), "w") as f:
        json.dump(hf_config(model.args), f, indent=2)
    return files


def hf_config(a) -> dict:
    cfg = {"architectures": ["Qwen3MoeForCausalLM" if a.num_experts else ("Qwen3ForCausalLM" if a.qk_norm
                                                                           else "LlamaForCausalLM")],
           "model_type": "qwen3_moe" if a.num_experts else ("qwen3" if a.qk_norm else "llama"),
           "vocab_size": a.vocab_size, "hidden_size": a.hidden_size, "num_hidden_layers": a.num_layers,
           "num_attention_heads": a.num_heads, "num_key_value_heads": a.num_kv_heads, "head_dim": a.head_dim,
           "intermediate_size": a.intermediate_size, "rms_norm_eps": a.rms_norm_eps, "rope_theta": a.rope_theta,
           "rope_scaling": a.rope_scaling, "tie_word_embeddings": a.tie_word_embeddings,
           "max_position_embeddings": a.max_position_embeddings, "hidden_act": "silu", "torch_dtype": "bfloat16",
           "attention_bias": False}
    if a.num_experts:
        cfg.update({"num_experts": a.num_experts, "num_experts_per_tok": a.num_experts_per_tok,
                    "moe_intermediate_size": a.moe_intermediate_size, "norm_topk_prob": a.norm_topk_prob,
                    "router_aux_loss_coef": a.router_aux_loss_coef, "decoder_sparse_step": a.decoder_sparse_step,
                    "mlp_only_layers": list(a.mlp_only_layers)})
    return cfg


def load_hf_safetensors(model, path: str, strict: bool = True) -> list[str]:
    """Load HF-named safetensors (a directory with an index, or one file)."""
    from safetensors.torch import load_file
    files = []
    if os.path.isdir(path):
        idx = os.path.join(path, "model.safetensors.index.json")
        if os.path.isfile(idx):
            with open(idx) as f:
                files = sorted(set(json.load(f)["weight_map"].values()))
        else:
            files = sorted(n for n in os.listdir(path) if n.endswith(".safetensors"))
        files = [os.path.join(path, n) for n in files]
    else:
        files = [path]
    sd: dict = {}
    for fp in files:
        sd.update(load_file(fp))
    return model.load_hf_state_dict(sd, strict=strict)


class CheckpointManager:
    """Keeps at most ``save_total_limit`` step directories under ``root``."""

    def __init__(self, root: str, save_total_limit: int = 3) -> None:
        self.root, self.limit = root, save_total_limit

    def steps(self) -> list[int]:
        if not os.path.isdir(self.root):
            return []
        return sorted(int(m.group(1)) for n in os.listdir(self.root) if (m := re.fullmatch(r"global_step_(\d+)", n)))

    def prune(self, keep_extra: int = 0) -> list[int]:
        st = self.steps()
        drop = st[: max(0, len(st) - max(self.limit - keep_extra, 0))] if self.limit > 0 else []
        for s in drop:
            shutil.rmtree(os.path.join(self.root, f"global_step_{s}"), ignore_errors=True)
        return drop

    def save(self, engine, step: int, rank: int = 0, world: int = 1, extra: Optional[dict] = None) -> str:
        self.prune(keep_extra=1)
        return save_sharded(engine, self.root, step, rank, world, extra)

    def load_latest(self, engine, rank: int = 0, world: int = 1, data=None) -> int:
        return load_sharded(engine, self.root, rank, world, data=data)
