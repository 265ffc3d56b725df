"""Training-inference separation with FSDP-style full sharding on the trainer
side (``policy.training.fsdp_cfg.reshard_after_forward``): 2 trainer ranks
holding half of the weights each + 1 rollout rank (gloo, CPU) produce the
same metrics and the same rollout weights as the unsharded run."""

import os

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from lumenrl_b200.core.config import LumenRLConfig
from lumenrl_b200.models.config import tiny_qwen3
from lumenrl_b200.parallel.dist import ParallelState
from lumenrl_b200.trainer.rl_trainer import RLRunSpec

HERE = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
STEPS = 2


def _worker(rank, world, port, q, shard):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from lumenrl_b200.engine.training.fsdp import ShardedParamActorEngine
        from lumenrl_b200.trainer.separated_trainer import SeparatedRLTrainer
        torch.manual_seed(0)
        cfg = LumenRLConfig.from_yaml(os.path.join(HERE, "configs", "grpo_tiny_cpu.yaml"),
                                      [f"num_training_steps={STEPS}", "policy.learning_rate=1e-3"])
        if shard:
            cfg.policy.training.fsdp_cfg = {"reshard_after_forward": True}
        spec = RLRunSpec(prompts_per_step=4, prompt_len=16, max_new_tokens=12, reward="contains_token",
                         eos_token_id=None)
        tr = SeparatedRLTrainer(cfg, tiny_qwen3(), spec, ParallelState(rank=rank, world_size=world),
                                num_rollout=1).setup()
        if not tr.is_rollout:
            assert isinstance(tr.actor, ShardedParamActorEngine) == shard
        hist = [tr.step() for _ in range(STEPS)]
        out = None if tr.is_rollout else [(m["reward/mean"], m["actor/grad_norm"]) for m in hist]
        q.put((rank, out, tr.model.flat.clone().numpy() if tr.is_rollout else None))
        dist.barrier()
        tr.close()
    except Exception as e:
        import traceback
        q.put((rank, "error: " + traceback.format_exc()[-2000:] + repr(e), None))
    dist.destroy_process_group()


def _run(shard: bool, port: int):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 3, port, q, shard)) for r in range(3)]
    for p in procs:
        p.start()
    res = {r: (m, w) for r, m, w in (q.get(timeout=900) for _ in procs)}
    for p in procs:
        p.join(timeout=60)
    for r, (m, _) in res.items():
        assert not (isinstance(m, str) and m.startswith("error")), m
    return res


def test_separated_with_sharded_trainer_matches_unsharded():
    base = 29900 + os.getpid() % 50
    a = _run(False, base)
    b = _run(True, base + 60)
    for r in (0, 1):                      # trainer ranks
        for (ra, ga), (rb, gb) in zip(a[r][0], b[r][0]):
            assert abs(ra - rb) < 1e-6 and abs(ga - gb) < 1e-4 * max(ga, 1e-6), (r, ra, rb, ga, gb)
    wa, wb = torch.from_numpy(a[2][1]), torch.from_numpy(b[2][1])   # rollout rank's weights
    assert (wa - wb).abs().max().item() < 1e-4
