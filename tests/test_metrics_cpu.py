"""Step metrics keep the reference's names (``rl_trainer.py:3427-3506,
3630-3652``; ``metric_utils.py:64-224``) and the mismatch diagnostics are
exact token- and sequence-weighted means that add up across ranks."""

import os

import torch

from lumenrl_b200.algorithms import rollout_correction as rc

HERE = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

REFERENCE_NAMES = [
    "timing/step_s", "timing/gen_s", "timing/train_s", "timing/weight_sync_s", "perf/throughput",
    "perf/gen_tokens_per_s", "perf/total_num_tokens", "reward/mean", "response_length/mean", "actor/entropy",
    "actor/grad_norm", "actor/pg_loss", "actor/pg_clipfrac", "actor/ppo_kl", "rollout_corr/kl",
    "rollout_corr/k3_kl", "rollout_corr/chi2_token", "rollout_corr/chi2_seq", "mismatch/abs_diff",
    "mismatch/k3_kl", "mismatch/chi2_token", "mismatch/chi2_seq", "mismatch/frac_abs_gt_0.1",
]
OWN_NAMES = ["perf/step_tokens_per_s", "weight_sync/ms", "weight_sync/GBps"]


def test_grpo_step_emits_reference_metric_names():
    from lumenrl_b200.core.config import LumenRLConfig
    from lumenrl_b200.models.config import tiny_llama
    from lumenrl_b200.parallel.dist import ParallelState
    from lumenrl_b200.trainer.metrics import with_aliases
    from lumenrl_b200.trainer.rl_trainer import RLRunSpec, RLTrainer
    cfg = LumenRLConfig.from_yaml(os.path.join(HERE, "configs", "grpo_tiny_cpu.yaml"), ["num_training_steps=1"])
    spec = RLRunSpec(prompts_per_step=4, prompt_len=16, max_new_tokens=16, reward="contains_token",
                     eos_token_id=None)
    m = RLTrainer(cfg, tiny_llama(), spec, ParallelState()).setup().step()
    absent = [k for k in REFERENCE_NAMES + OWN_NAMES if k not in m]
    assert not absent, absent
    aliased = with_aliases(m)
    assert "critic/score/mean" in aliased and "timing_s/step" in aliased
    # rollout and training forwards agree on the same weights: no mismatch tail
    assert m["mismatch/frac_abs_gt_0.1"] == 0.0 and m["mismatch/abs_diff"] < 1e-2


def test_mismatch_sums_are_exact_and_additive():
    g = torch.Generator().manual_seed(0)
    B, S = 6, 20
    train = -torch.rand(B, S, generator=g, dtype=torch.float64) * 3
    roll = train + 0.2 * torch.randn(B, S, generator=g, dtype=torch.float64)
    mask = (torch.arange(S)[None] < torch.randint(5, S + 1, (B, 1), generator=g)).double()
    got = rc.finalize_mismatch(rc.mismatch_sums(train, roll, mask).tolist())
    r = (train - roll) * mask
    w = torch.exp(r)
    tok = mask.sum()
    want = {"mismatch/abs_diff": r.abs().sum() / tok, "mismatch/k3_kl": ((w - 1 - r) * mask).sum() / tok,
            "mismatch/chi2_token": ((w - 1) ** 2 * mask).sum() / tok,
            "mismatch/frac_abs_gt_0.1": ((r.abs() > 0.1).double() * mask).sum() / tok,
            "mismatch/chi2_seq": ((torch.exp(r.sum(-1)) - 1) ** 2).mean()}
    for k, v in want.items():
        assert abs(got[k] - float(v)) < 1e-9 * max(1.0, abs(float(v))), k
    # two ranks' sums add up to the whole batch's
    halves = rc.mismatch_sums(train[:2], roll[:2], mask[:2]) + rc.mismatch_sums(train[2:], roll[2:], mask[2:])
    whole = rc.finalize_mismatch(halves.tolist())
    assert all(abs(whole[k] - got[k]) < 1e-12 for k in got)


def test_profiler_traces_the_selected_step(tmp_path):
    from lumenrl_b200.core.config import LumenRLConfig
    from lumenrl_b200.models.config import tiny_llama
    from lumenrl_b200.parallel.dist import ParallelState
    from lumenrl_b200.trainer.rl_trainer import RLRunSpec, RLTrainer
    out = str(tmp_path / "prof")
    cfg = LumenRLConfig.from_yaml(os.path.join(HERE, "configs", "grpo_tiny_cpu.yaml"),
                                  ["num_training_steps=2", "profiler.enable=true", "profiler.tool=torch",
                                   f"profiler.save_path={out}", "profiler.steps=[1]"])
    spec = RLRunSpec(prompts_per_step=2, prompt_len=8, max_new_tokens=8, reward="contains_token", eos_token_id=None)
    tr = RLTrainer(cfg, tiny_llama(), spec, ParallelState()).setup()
    tr.step()
    assert getattr(tr, "last_trace", None) is None          # step 0 is not profiled
    tr.step()
    assert tr.last_trace == os.path.join(out, "trace_rank0_step1.json") and os.path.getsize(tr.last_trace) > 0


def test_dashboard_renders_charts_from_metric_logs(tmp_path):
    import json

    from lumenrl_b200.utils.dashboard import load_records, render_dashboard
    p = tmp_path / "metrics.jsonl"
    with open(p, "w") as f:
        for s in range(1, 6):
            f.write(json.dumps({"step": s, "reward/mean": 0.1 * s, "timing/step_s": 11.0 + 0.01 * s,
                                "weight_sync/ms": 41.0}) + "\n")
    out = tmp_path / "dash.html"
    drawn = render_dashboard(load_records([str(p)]), str(out))
    assert drawn == ["reward/mean", "timing/step_s", "weight_sync/ms"]
    text = out.read_text()
    assert text.count("<svg") == 3 and "<script" not in text and "0.5" in text


def _reduce_worker(rank, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE="2")
    from lumenrl_b200.parallel.dist import all_reduce_max_many, all_reduce_sum_many, init_distributed
    init_distributed(backend="gloo", timeout_s=30.0, device="cpu")
    vals = [1.0 + rank, 10.0 * rank, -3.0 + rank]
    q.put((rank, all_reduce_sum_many(vals), all_reduce_max_many(vals), all_reduce_sum_many([])))
    dist.barrier()
    dist.destroy_process_group()


def test_vector_reductions_over_two_ranks():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29400 + os.getpid() % 200
    procs = [ctx.Process(target=_reduce_worker, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {r: (s, m, e) for r, s, m, e in (q.get(timeout=120) for _ in procs)}
    for p in procs:
        p.join(timeout=60)
    for r in (0, 1):
        assert res[r] == ([3.0, 10.0, -5.0], [2.0, 10.0, -2.0], [])
