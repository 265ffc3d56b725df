"""Colocated GRPO with rollout tensor parallelism (TP = 2 over 2 gloo ranks):
the TP group generates the single-process run's prompts and samples, each
member trains on every second GRPO group, and the updated weights equal the
single-process run's."""

import os

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from lumenrl_b200.core.config import LumenRLConfig
from lumenrl_b200.models.config import tiny_llama
from lumenrl_b200.parallel.dist import ParallelState
from lumenrl_b200.trainer.rl_trainer import RLRunSpec, RLTrainer

HERE = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
STEPS = 2


def _cfg(tp: int):
    return LumenRLConfig.from_yaml(os.path.join(HERE, "configs", "grpo_tiny_cpu.yaml"),
                                   ["algorithm.name=grpo", f"policy.generation.vllm_cfg.tensor_parallel_size={tp}"])


def _spec():
    return RLRunSpec(prompts_per_step=4, prompt_len=16, max_new_tokens=12, reward="contains_token", eos_token_id=None)


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.manual_seed(0)
    tr = RLTrainer(_cfg(2), tiny_llama(), _spec(), ParallelState(rank=rank, world_size=world)).setup()
    assert tr.rollout.tp is not None and tr.rollout.cache.spec.num_kv_heads == tr.model_args.num_kv_heads // 2
    hist = [tr.step() for _ in range(STEPS)]
    q.put((rank, [m["reward/mean"] for m in hist], tr.actor.model.flat.clone()))
    dist.barrier()
    dist.destroy_process_group()


def test_grpo_with_rollout_tp2_matches_single_process():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29450 + os.getpid() % 300
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict((r, (rw, w)) for r, rw, w in (q.get(timeout=600) for _ in procs))
    for p in procs:
        p.join(timeout=60)
    torch.manual_seed(0)
    single = RLTrainer(_cfg(1), tiny_llama(), _spec(), ParallelState()).setup()
    ref = [single.step() for _ in range(STEPS)]
    for r in (0, 1):
        rewards, w = res[r]
        for a, m in zip(rewards, ref):
            assert abs(a - m["reward/mean"]) < 1e-6, (r, a, m["reward/mean"])
        assert torch.allclose(w.float(), single.actor.model.flat.float(), atol=1e-5), r
