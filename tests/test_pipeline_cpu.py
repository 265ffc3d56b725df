"""Pipeline parallelism (1F1B over gloo point-to-point) on 2 and 3 CPU
ranks: the summed loss and every parameter gradient equal a single-process
run over the same micro-batches (fp32)."""

import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _batches(args, n_mb, seed=0):
    from lumenrl_b200.parallel.pipeline import MicroBatch
    g = torch.Generator().manual_seed(seed)
    out = []
    for i in range(n_mb):
        lens = [5 + (3 * i) % 7, 9 + i % 4]
        T = sum(lens)
        ids = torch.randint(0, args.vocab_size, (T,), generator=g)
        out.append(MicroBatch(ids=ids, positions=torch.cat([torch.arange(n) for n in lens]),
                              cu=torch.tensor([0, lens[0], T], dtype=torch.int32), max_len=max(lens),
                              targets=torch.randint(0, args.vocab_size, (T,), generator=g),
                              weights=torch.rand(T, generator=g)))
    return out


def _model():
    from lumenrl_b200.models.config import tiny_llama
    from lumenrl_b200.models.qwen3 import Qwen3Model
    m = Qwen3Model(tiny_llama(), dtype=torch.float32, requires_grad=True)
    m.init_weights(3)
    return m


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from lumenrl_b200.parallel.pipeline import OneFOneB, PipelineStage, embedding_group
    m = _model()
    ends = embedding_group(world)
    st = PipelineStage(m, rank, world)
    loss = OneFOneB(st, torch.device("cpu"), torch.float32).run(_batches(m.args, 5), loss_scale=0.5)
    st.sync_tied_embedding_grad(ends)   # tiny_llama ties the embedding and the LM head
    # numpy arrays travel by value (tensors would travel as shared-memory handles
    # that vanish when this process exits)
    grads = {n: p.grad.numpy().copy() for n, p in m.named_flat_params() if p.grad is not None}
    q.put((rank, loss, grads, [n for n, p in m.named_flat_params() if any(p is x for x in st.params())]))
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_1f1b_matches_single_process(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29200 + 10 * world + os.getpid() % 90
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {r: (l, g, names) for r, l, g, names in (q.get(timeout=300) for _ in procs)}
    for p in procs:
        p.join(timeout=60)
    # single-process reference over the same micro-batches
    from lumenrl_b200.parallel.pipeline import PipelineStage
    m = _model()
    st = PipelineStage(m, 0, 1)
    total = 0.0
    for mb in _batches(m.args, 5):
        loss = st.loss(mb, st.forward(mb, None)) * 0.5
        loss.backward()
        total += float(loss)
    assert abs(res[world - 1][0] - total) < 1e-4 * max(1.0, abs(total))
    ref = {n: p.grad for n, p in m.named_flat_params()}
    seen = set()
    for r, (_, grads, names) in res.items():
        for n in names:
            assert n in grads, (r, n)
            assert torch.allclose(torch.from_numpy(grads[n]), ref[n], atol=1e-5, rtol=1e-4), (r, n)
            seen.add(n)
    assert seen == set(ref)   # every parameter is owned by some stage
