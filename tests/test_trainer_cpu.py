"""BASELINE config 0 on CPU: tiny Llama GRPO, 3 steps; gloo world_size=2
sharded optimizer equals the single-process update."""

import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from lumenrl_b200.core.config import LumenRLConfig
from lumenrl_b200.engine.training.optimizer import ShardedFlatAdamW
from lumenrl_b200.models.config import tiny_llama
from lumenrl_b200.parallel.dist import ParallelState
from lumenrl_b200.trainer.rl_trainer import RLRunSpec, RLTrainer

HERE = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _cfg(algo="grpo"):
    return LumenRLConfig.from_yaml(os.path.join(HERE, "configs", "grpo_tiny_cpu.yaml"),
                                   [f"algorithm.name={algo}", "algorithm.dapo.num_generations=4"])


@pytest.mark.parametrize("algo", ["grpo", "dapo"])
def test_three_step_grpo_cpu(algo):
    torch.manual_seed(0)
    spec = RLRunSpec(prompts_per_step=8, prompt_len=32, max_new_tokens=32, reward="contains_token",
                     eos_token_id=None)
    tr = RLTrainer(_cfg(algo), tiny_llama(), spec, ParallelState()).setup()
    w0 = tr.actor.model.flat.clone()
    hist = tr.train()
    assert len(hist) == 3
    for m in hist:
        assert m["perf/total_num_tokens"] == 8 * 4 * (32 + 32)
        assert abs(m["rollout_corr/kl"]) < 1e-3   # rollout and training forwards agree
    assert any(m["actor/grad_norm"] > 0 for m in hist)
    assert not torch.equal(w0, tr.actor.model.flat)


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.manual_seed(0)
    n = 1024
    w = torch.randn(n)
    opt = ShardedFlatAdamW(w.clone(), world, rank, lr=1e-2, betas=(0.9, 0.95), weight_decay=0.1, max_grad_norm=1.0)
    for step in range(3):
        g = torch.randn(n, generator=torch.Generator().manual_seed(100 * step + rank))
        opt.grad.copy_(g)
        st = opt.step()
    q.put((rank, opt.w16.clone(), st["grad_norm"]))
    dist.destroy_process_group()


def test_sharded_optimizer_matches_single_process():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + os.getpid() % 200
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=120) for _ in procs], key=lambda x: x[0])
    for p in procs:
        p.join(timeout=60)
    torch.manual_seed(0)
    n = 1024
    w = torch.randn(n)
    single = ShardedFlatAdamW(w.clone(), 1, 0, lr=1e-2, betas=(0.9, 0.95), weight_decay=0.1, max_grad_norm=1.0)
    for step in range(3):
        g = sum(torch.randn(n, generator=torch.Generator().manual_seed(100 * step + r)) for r in range(2))
        single.grad.copy_(g)
        s = single.step()
    assert torch.allclose(res[0][1], single.w16, atol=1e-6)
    assert torch.allclose(res[1][1], single.w16, atol=1e-6)
    assert abs(res[0][2] - s["grad_norm"]) < 1e-3


def test_ppo_with_critic_three_steps_cpu():
    """PPO: critic values feed GAE, the policy and the critic both update."""
    torch.manual_seed(0)
    cfg = LumenRLConfig.from_yaml(os.path.join(HERE, "configs", "grpo_tiny_cpu.yaml"),
                                  ["algorithm.name=ppo", "algorithm.ppo.num_mini_batches=2",
                                   "algorithm.ppo.num_ppo_epochs=1", "critic.learning_rate=1e-3"])
    spec = RLRunSpec(prompts_per_step=8, prompt_len=16, max_new_tokens=16, reward="contains_token",
                     eos_token_id=None)
    tr = RLTrainer(cfg, tiny_llama(), spec, ParallelState()).setup()
    assert tr.critic is not None and tr.ref is not None
    c0 = tr.critic.model.flat.clone()
    head0 = tr.critic.head.weight.detach().clone()
    hist = tr.train()
    assert len(hist) == 3
    for m in hist:
        assert "critic/vf_loss" in m and m["critic/vf_loss"] == m["critic/vf_loss"]
        assert "timing/values_s" in m and "timing/critic_s" in m
    assert not torch.equal(c0, tr.critic.model.flat) or not torch.equal(head0, tr.critic.head.weight)


def test_dapo_refill_rounds_collect_informative_groups_cpu():
    """DAPO filter_groups: rounds repeat until enough groups with non-constant
    rewards are kept; every kept group has reward variance."""
    torch.manual_seed(0)
    cfg = LumenRLConfig.from_yaml(os.path.join(HERE, "configs", "grpo_tiny_cpu.yaml"),
                                  ["algorithm.name=dapo", "algorithm.dapo.num_generations=4",
                                   "algorithm.dapo.filter_groups.enable=true",
                                   "algorithm.dapo.filter_groups.max_num_gen_batches=6"])
    spec = RLRunSpec(prompts_per_step=4, prompt_len=16, max_new_tokens=16, reward="contains_token",
                     eos_token_id=None)
    tr = RLTrainer(cfg, tiny_llama(), spec, ParallelState()).setup()
    # reward 1 when the first response token is a multiple of 5 (p ~ 0.2): about
    # 40 % of 4-sample groups are all-zero, so refill rounds are needed
    tr.reward_fn = lambda responses, prompts=None, lengths=None, **_: (responses[:, 0] % 5 == 0).float()
    seen = []
    orig = tr._rollout

    def spy(step, round_idx=0):
        b = orig(step, round_idx)
        seen.append(round_idx)
        return b
    tr._rollout = spy
    hist = tr.train()
    assert len(hist) == 3
    assert max(seen) >= 1                       # at least one refill round ran
    for m in hist:
        assert 1 <= m["dapo/gen_rounds"] <= 6
        assert m["dapo/kept_groups"] <= 4


def test_kl_in_reward_uses_reference_and_controller_cpu():
    torch.manual_seed(0)
    cfg = LumenRLConfig.from_yaml(os.path.join(HERE, "configs", "grpo_tiny_cpu.yaml"),
                                  ["algorithm.use_kl_in_reward=true", "algorithm.grpo.kl_coeff=0.05",
                                   "algorithm.kl_ctrl_type=adaptive"])
    spec = RLRunSpec(prompts_per_step=8, prompt_len=16, max_new_tokens=16, reward="contains_token",
                     eos_token_id=None)
    tr = RLTrainer(cfg, tiny_llama(), spec, ParallelState()).setup()
    assert tr.kl_ctrl is not None and tr.ref is not None
    hist = tr.train()
    for m in hist:
        assert "actor/reward_kl_penalty" in m and "actor/reward_kl_penalty_coeff" in m
    # the policy moves away from the frozen reference, so later steps see a KL
    assert hist[-1]["actor/reward_kl_penalty"] != 0.0


def test_dapo_fp8_recipe_runs_cpu():
    """Config 2 plumbing: W8A8 FP8 rollout + hybrid FP8 training linears."""
    torch.manual_seed(0)
    cfg = LumenRLConfig.from_yaml(os.path.join(HERE, "configs", "grpo_tiny_cpu.yaml"),
                                  ["algorithm.name=dapo", "algorithm.dapo.num_generations=4",
                                   "quantization.training.fp8=hybrid", "quantization.rollout.precision=fp8",
                                   "quantization.rollout_correction.rollout_is=token",
                                   "quantization.rollout_correction.rollout_is_threshold=2.0", "num_training_steps=1"])
    spec = RLRunSpec(prompts_per_step=4, prompt_len=16, max_new_tokens=16, reward="contains_token",
                     eos_token_id=None)
    tr = RLTrainer(cfg, tiny_llama(), spec, ParallelState()).setup()
    assert tr.actor.model.fp8_training is tr.fp8_training and tr.fp8_training.enabled
    assert tr.rollout.runner.fp8 is not None
    calls = {"n": 0}
    orig = tr.fp8_training.linear

    def spy(*a, **k):
        calls["n"] += 1
        return orig(*a, **k)
    tr.fp8_training.linear = spy
    hist = tr.train()
    assert calls["n"] > 0
    for m in hist:
        assert m["actor/grad_norm"] == m["actor/grad_norm"]
        assert "rollout_corr/kl" in m
