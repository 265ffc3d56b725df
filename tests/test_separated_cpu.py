"""Training-inference separation on CPU ranks (gloo): one trainer rank and
one rollout rank (weights broadcast after every step, rollout rows and the
MoE routed-expert ids sent to the trainer) reproduce the colocated
single-process run of the same tiny MoE model, step for step."""

import os

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from lumenrl_b200.core.config import LumenRLConfig
from lumenrl_b200.models.config import tiny_qwen3_moe
from lumenrl_b200.parallel.dist import ParallelState
from lumenrl_b200.trainer.rl_trainer import RLRunSpec, RLTrainer

HERE = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
STEPS = 2


def _cfg():
    return LumenRLConfig.from_yaml(os.path.join(HERE, "configs", "grpo_tiny_cpu.yaml"),
                                   [f"num_training_steps={STEPS}", "policy.learning_rate=1e-3"])


def _spec():
    return RLRunSpec(prompts_per_step=4, prompt_len=16, max_new_tokens=12, reward="contains_token",
                     eos_token_id=None)


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from lumenrl_b200.trainer.separated_trainer import SeparatedRLTrainer
    torch.manual_seed(0)
    tr = SeparatedRLTrainer(_cfg(), tiny_qwen3_moe(), _spec(), ParallelState(rank=rank, world_size=world),
                            num_rollout=1).setup()
    hist = [tr.step() for _ in range(STEPS)]
    if tr.is_rollout:
        q.put((rank, None, tr.model.flat.clone()))
    else:
        q.put((rank, [(m["reward/mean"], m["actor/pg_loss"], m["actor/grad_norm"]) for m in hist],
               tr.model.flat.clone()))
    dist.barrier()
    tr.close()
    dist.destroy_process_group()


def test_separated_matches_colocated_moe_with_routing_replay():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29550 + os.getpid() % 200
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {r: (m, w) for r, m, w in (q.get(timeout=300) for _ in procs)}
    for p in procs:
        p.join(timeout=60)
    torch.manual_seed(0)
    single = RLTrainer(_cfg(), tiny_qwen3_moe(), _spec(), ParallelState()).setup()
    ref = [single.step() for _ in range(STEPS)]
    sep_metrics, sep_w = res[0]
    for (r, l, g), m in zip(sep_metrics, ref):
        assert abs(r - m["reward/mean"]) < 1e-6
        assert abs(l - m["actor/pg_loss"]) < 1e-4 * max(1.0, abs(m["actor/pg_loss"]))
        assert abs(g - m["actor/grad_norm"]) < 1e-4 * max(1.0, m["actor/grad_norm"])
    assert torch.allclose(sep_w, single.actor.model.flat, atol=1e-6)
    # the rollout rank holds the trainer's latest weights
    assert torch.equal(res[1][1], sep_w)


def _async_worker(rank, world, port, q, lag):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from lumenrl_b200.trainer.separated_trainer import SeparatedRLTrainer
    torch.manual_seed(0)
    cfg = LumenRLConfig.from_yaml(os.path.join(HERE, "configs", "grpo_tiny_cpu.yaml"),
                                  ["num_training_steps=3", "policy.learning_rate=3e-3"])
    from lumenrl_b200.models.config import tiny_llama
    tr = SeparatedRLTrainer(cfg, tiny_llama(), _spec(), ParallelState(rank=rank, world_size=world), num_rollout=1,
                            async_lag=lag).setup()
    hist = []
    for _ in range(3):
        hist.append(tr.step())
        dist.barrier()      # a barrier between steps (bench.py's timed-region boundary) must not deadlock
    tr.finish()
    q.put((rank, [m.get("rollout_corr/kl") for m in hist] if not tr.is_rollout else None, tr.model.flat.clone()))
    dist.barrier()
    tr.close()
    dist.destroy_process_group()


def test_async_separated_is_one_step_stale():
    """async_lag=1: the rollout generates batch s+1 while batch s trains, so
    from the second step on the trainer sees rollout log-probs of the previous
    policy (non-zero rollout/training KL); synchronous runs see none.  After
    finish() the rollout holds the trainer's final weights in both modes."""
    ctx = mp.get_context("spawn")
    kls = {}
    for lag in (0, 1):
        q = ctx.Queue()
        port = 29650 + os.getpid() % 150 + 7 * lag
        procs = [ctx.Process(target=_async_worker, args=(r, 2, port, q, lag)) for r in range(2)]
        for p in procs:
            p.start()
        res = {r: (k, w) for r, k, w in (q.get(timeout=300) for _ in procs)}
        for p in procs:
            p.join(timeout=60)
        kls[lag] = res[0][0]
        assert torch.equal(res[0][1], res[1][1])
    assert all(abs(k) < 1e-4 for k in kls[0]), kls
    assert abs(kls[1][0]) < 1e-4 and all(abs(k) > 1e-5 for k in kls[1][1:]), kls
