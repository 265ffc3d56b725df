"""Parameter-sharded training engine (ZeRO-3 / FSDP-style) on 2 gloo CPU
ranks against the unsharded single-process engine: the same initial model,
the same scored log-probs, the same global gradient norm and the same update
after a GRPO step on the union of the ranks' batches."""

import os

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _batch(seed: int):
    from lumenrl_b200.core.protocol import DataProto
    g = torch.Generator().manual_seed(seed)
    B, P, R = 4, 12, 9
    plen = torch.randint(5, P + 1, (B,), generator=g)
    rlen = torch.randint(3, R + 1, (B,), generator=g)
    mask = (torch.arange(R).unsqueeze(0) < rlen.unsqueeze(1)).float()
    return DataProto({"prompt_ids": torch.randint(3, 2048, (B, P), generator=g), "prompt_lengths": plen,
                      "responses": torch.randint(3, 2048, (B, R), generator=g), "response_lengths": rlen,
                      "response_mask": mask, "old_log_probs": -torch.rand(B, R, generator=g) * 8,
                      "advantages": torch.randn(B, generator=g)})


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from lumenrl_b200.core.config import GRPOConfig
        from lumenrl_b200.engine.training.fsdp import ShardedParamActorEngine
        from lumenrl_b200.models.config import tiny_qwen3
        from lumenrl_b200.parallel.dist import ParallelState
        eng = ShardedParamActorEngine(tiny_qwen3(), ParallelState(world_size=world, rank=rank), lr=1e-3, seed=3)
        w0 = eng.full_flat()
        b = _batch(rank)
        lp, ent = eng.compute_log_probs(b)
        gn = eng.update_policy(b, GRPOConfig(), "grpo", rows_per_micro=2)["actor/grad_norm"]
        # numpy copies travel by value (tensors would be shared through file
        # descriptors that disappear when this process exits)
        q.put((rank, {"w0": w0.numpy(), "lp": lp.numpy(), "ent": ent.numpy(), "gn": gn,
                      "w1": eng.full_flat().numpy(), "shard_numel": eng.w16.numel()}))
    except Exception as e:  # surfaced by the parent
        import traceback
        q.put((rank, {"error": traceback.format_exc()[-2000:] + repr(e)}))
    dist.destroy_process_group()


def test_sharded_params_match_unsharded_engine():
    from lumenrl_b200.core.config import GRPOConfig
    from lumenrl_b200.core.protocol import DataProto
    from lumenrl_b200.engine.training.actor import ActorEngine
    from lumenrl_b200.models.config import tiny_qwen3
    from lumenrl_b200.parallel.dist import ParallelState
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29810 + os.getpid() % 150
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=600) for _ in procs)
    for r in res.values():
        for k in ("w0", "lp", "ent", "w1"):
            if k in r:
                r[k] = torch.from_numpy(r[k])
    for p in procs:
        p.join(timeout=60)
    for r in (0, 1):
        assert "error" not in res[r], res[r]["error"]
    ref = ActorEngine(tiny_qwen3(), ParallelState(), lr=1e-3, seed=3)
    n = ref.model.layout.numel
    w0 = ref.model.flat[:n].clone()
    assert torch.equal(res[0]["w0"][:n], w0) and torch.equal(res[1]["w0"][:n], w0)
    # each rank holds about half of the weights
    assert res[0]["shard_numel"] < 0.6 * n
    both = DataProto.concat([_batch(0), _batch(1)])
    lp, ent = ref.compute_log_probs(both)
    m = both.tensors["response_mask"] > 0
    for r in (0, 1):
        rows = slice(4 * r, 4 * r + 4)
        assert float((res[r]["lp"] - lp[rows])[m[rows]].abs().max()) < 1e-4
        assert float((res[r]["ent"] - ent[rows])[m[rows]].abs().max()) < 1e-4
    gn = ref.update_policy(both, GRPOConfig(), "grpo", rows_per_micro=2)["actor/grad_norm"]
    assert abs(res[0]["gn"] - gn) < 1e-4 * gn and abs(res[1]["gn"] - gn) < 1e-4 * gn
    moved = float((ref.model.flat[:n] - w0).abs().max())
    assert moved > 1e-4
    for r in (0, 1):
        # Adam's first step is ~lr * sign(g): weights whose gradient is at the
        # rounding level may differ by a fraction of one step, no more
        assert float((res[r]["w1"][:n] - ref.model.flat[:n]).abs().max()) < 0.1 * moved


def test_sft_with_fsdp_cfg_uses_sharded_engine_and_matches():
    """policy.training.fsdp_cfg.reshard_after_forward selects the sharded engine
    in SFT; two steps give the losses of the resident-weight engine."""
    from lumenrl_b200.core.config import LumenRLConfig
    from lumenrl_b200.core.protocol import DataProto
    from lumenrl_b200.engine.training.fsdp import ShardedParamActorEngine
    from lumenrl_b200.models.config import tiny_llama
    from lumenrl_b200.parallel.dist import ParallelState
    from lumenrl_b200.trainer.sft_trainer import SFTTrainer
    here = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    b = DataProto({"prompt_ids": torch.randint(3, 2048, (4, 8), generator=torch.Generator().manual_seed(0)),
                   "prompt_lengths": torch.full((4,), 8),
                   "responses": torch.randint(3, 2048, (4, 6), generator=torch.Generator().manual_seed(1)),
                   "response_lengths": torch.tensor([6, 5, 4, 6]),
                   "response_mask": (torch.arange(6).unsqueeze(0) < torch.tensor([6, 5, 4, 6]).unsqueeze(1)).float()})
    losses = {}
    for shard in (False, True):
        cfg = LumenRLConfig.from_yaml(os.path.join(here, "configs", "grpo_tiny_cpu.yaml"),
                                      ["policy.learning_rate=1e-3"])
        if shard:
            cfg.policy.training.fsdp_cfg = {"reshard_after_forward": True}
        sft = SFTTrainer(cfg, tiny_llama(), ParallelState())
        assert isinstance(sft.engine, ShardedParamActorEngine) == shard
        losses[shard] = [sft.step(b)["sft/loss"] for _ in range(2)]
    for a, c in zip(losses[False], losses[True]):
        assert abs(a - c) < 1e-5 * max(1.0, abs(a)), losses
