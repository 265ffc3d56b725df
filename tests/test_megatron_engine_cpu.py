"""Megatron-style engine on 4 CPU ranks (gloo): TP=2 x PP=2 with sequence
parallelism and 1F1B; the loss and every gradient equal a single-process run
of the full model over the same micro-batches (fp32)."""

import os

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _batches(vocab, n_mb, seed=0):
    from lumenrl_b200.parallel.pipeline import MicroBatch
    g = torch.Generator().manual_seed(seed)
    out = []
    for i in range(n_mb):
        lens = [6 + 2 * (i % 3), 10]
        T = sum(lens)
        out.append(MicroBatch(ids=torch.randint(0, vocab, (T,), generator=g),
                              positions=torch.cat([torch.arange(n) for n in lens]),
                              cu=torch.tensor([0, lens[0], T], dtype=torch.int32), max_len=max(lens),
                              targets=torch.randint(0, vocab, (T,), generator=g), weights=torch.rand(T, generator=g)))
    return out


def _worker(rank, world, port, q, vocab_parallel=False):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from lumenrl_b200.engine.training.megatron_engine import MegatronEngine
    from lumenrl_b200.models.config import tiny_qwen3
    from lumenrl_b200.parallel.tensor_parallel import shard_cols, shard_gate_up, shard_qkv
    args = tiny_qwen3(layers=4)
    eng = MegatronEngine(args, tp=2, pp=2, seed=5, vocab_parallel=vocab_parallel)
    loss = eng.forward_backward(_batches(args.vocab_size, 3))
    eng.sync_grads()
    g = eng.g
    out = {"loss": loss, "stage": g["stage"], "t": g["t"], "lo": eng.layer_range[0], "grads": {},
           "vocab": (eng.vocab_start, eng.vocab_start + (eng.lm_head.shape[0] if eng.lm_head is not None else 0))}
    for j, layer in enumerate(eng.layers):
        for name in ("wqkv", "wo", "w13", "w2", "ln1", "ln2", "q_norm", "k_norm"):
            out["grads"][f"{eng.layer_range[0] + j}.{name}"] = getattr(layer, name).grad.numpy().copy()
    for name in ("embed", "norm", "lm_head"):
        p = getattr(eng, name)
        if p is not None:
            out["grads"][name] = p.grad.numpy().copy()
    q.put((rank, out))
    dist.barrier()
    dist.destroy_process_group()


import pytest  # noqa: E402


@pytest.mark.parametrize("vocab_parallel", [False, True])
def test_tp2_pp2_matches_single_process(vocab_parallel):
    """vocab_parallel=True: the LM head split by rows over the TP group."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29100 + os.getpid() % 90 + (300 if vocab_parallel else 0)
    procs = [ctx.Process(target=_worker, args=(r, 4, port, q, vocab_parallel)) for r in range(4)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    from lumenrl_b200.models.config import tiny_qwen3
    from lumenrl_b200.models.qwen3 import Qwen3Model
    from lumenrl_b200.parallel.pipeline import PipelineStage
    from lumenrl_b200.parallel.tensor_parallel import shard_cols, shard_gate_up, shard_qkv
    args = tiny_qwen3(layers=4)
    m = Qwen3Model(args, dtype=torch.float32, requires_grad=True)
    m.init_weights(5)
    st = PipelineStage(m, 0, 1)
    total = 0.0
    for mb in _batches(args.vocab_size, 3):
        loss = st.loss(mb, st.forward(mb, None))
        loss.backward()
        total += float(loss)
    for r, out in res.items():
        assert abs(out["loss"] - total) < 1e-4 * max(1.0, abs(total)), (r, out["loss"], total)
    shard = {"wqkv": lambda g, t: shard_qkv(g, args.num_heads, args.num_kv_heads, args.head_dim, t, 2),
             "wo": lambda g, t: shard_cols(g, t, 2), "w13": lambda g, t: shard_gate_up(g, t, 2),
             "w2": lambda g, t: shard_cols(g, t, 2)}
    seen = set()
    for r, out in res.items():
        for key, got in out["grads"].items():
            if "." in key:
                i, name = key.split(".")
                ref = m.p(f"layers.{i}.{name}").grad
                if name in shard:
                    ref = shard[name](ref, out["t"])
            else:
                ref = m.p(key).grad if key != "lm_head" else m.lm_head.grad
                if key == "lm_head" and vocab_parallel:
                    ref = ref[out["vocab"][0]: out["vocab"][1]]
            assert np.allclose(got, ref.numpy(), atol=2e-5, rtol=1e-4), (r, key, np.abs(got - ref.numpy()).max())
            seen.add(key)
    assert {f"{i}.wqkv" for i in range(4)} <= seen and {"embed", "norm", "lm_head"} <= seen


def _step_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from lumenrl_b200.engine.training.megatron_engine import MegatronEngine
    from lumenrl_b200.models.config import tiny_llama
    args = tiny_llama()              # tied embeddings across the pipeline ends
    eng = MegatronEngine(args, tp=1, pp=2, seed=1, lr=3e-3)   # + DP 2
    losses = [eng.step(_batches(args.vocab_size, 2, seed=0))["loss"] for _ in range(4)]
    q.put((rank, losses))
    dist.barrier()
    dist.destroy_process_group()


def test_pp2_dp2_tied_embeddings_loss_decreases():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29010 + os.getpid() % 80
    procs = [ctx.Process(target=_step_worker, args=(r, 4, port, q)) for r in range(4)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for r, losses in res.items():
        assert losses[-1] < losses[0], (r, losses)
    assert all(abs(res[r][0] - res[0][0]) < 1e-6 for r in res)
