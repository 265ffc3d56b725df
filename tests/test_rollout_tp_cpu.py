"""Tensor-parallel rollout (TP = 2, gloo, CPU fp32) against the same engine
on one process: identical samples and rollout log-probs, and a weight sync
reaches the shards."""

import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _model():
    from lumenrl_b200.models.config import tiny_qwen3
    from lumenrl_b200.models.qwen3 import Qwen3Model
    m = Qwen3Model(tiny_qwen3(), dtype=torch.float32, requires_grad=False)
    m.init_weights(5)
    return m


def _generate(eng, bump: bool):
    from lumenrl_b200.engine.inference.engine import SamplingParams
    sp = SamplingParams(max_new_tokens=8, n=2, seed=3, stop_at_eos=False)
    out = [eng.generate([[5, 6, 7, 8, 9], [11, 12, 13]], sp)]
    if bump:   # a weight sync: every weight changes, the shards must follow
        with torch.no_grad():
            eng.model.flat.mul_(1.1)
        eng.update_weights()
        out.append(eng.generate([[5, 6, 7, 8, 9], [11, 12, 13]], sp))
    return [(o.responses.clone(), o.logprobs.clone()) for o in out]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from lumenrl_b200.engine.inference.engine import RolloutEngine
    eng = RolloutEngine(_model(), max_num_seqs=8, max_model_len=64, use_cuda_graph=False,
                        tp_group=dist.group.WORLD)
    assert eng.cache.spec.num_kv_heads == eng.args.num_kv_heads // world
    q.put((rank, _generate(eng, True)))
    dist.barrier()
    dist.destroy_process_group()


def test_rollout_tp2_matches_single_process():
    from lumenrl_b200.engine.inference.engine import RolloutEngine
    ref = _generate(RolloutEngine(_model(), max_num_seqs=8, max_model_len=64, use_cuda_graph=False), True)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29300 + os.getpid() % 500
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for rank in (0, 1):
        for (tok, lp), (rtok, rlp) in zip(res[rank], ref):
            assert torch.equal(tok, rtok), rank
            assert (lp - rlp).abs().max().item() < 1e-4, rank


def test_rollout_tp_rejects_indivisible_heads():
    from lumenrl_b200.engine.inference.runner import TPShards
    with pytest.raises(ValueError, match="must divide"):
        TPShards(_model(), None, 0, 3)
