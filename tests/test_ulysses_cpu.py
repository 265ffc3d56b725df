"""Ulysses sequence parallelism on 2 CPU ranks: attention over all-to-all
head shards equals full attention, forward and backward (fp32, GQA)."""

import os

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _data():
    g = torch.Generator().manual_seed(0)
    T, Hq, Hk, D = 24, 4, 2, 16
    q, k, v, do = (torch.randn(T, h, D, generator=g) for h in (Hq, Hk, Hk, Hq))
    cu = torch.tensor([0, 10, 24], dtype=torch.int32)
    return q, k, v, do, cu


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from lumenrl_b200.parallel.ulysses import ulysses_attention
    q, k, v, do, cu = _data()
    n = q.shape[0] // world
    sl = slice(rank * n, (rank + 1) * n)
    ql, kl, vl = (t[sl].clone().requires_grad_(True) for t in (q, k, v))
    o = ulysses_attention(ql, kl, vl, cu, 14, scale=0.25)
    o.backward(do[sl])
    out.put((rank, {n_: t.detach().numpy().copy() for n_, t in
                    (("o", o), ("dq", ql.grad), ("dk", kl.grad), ("dv", vl.grad))}))
    dist.destroy_process_group()


def test_ulysses_matches_full_attention():
    from lumenrl_b200.ops.reference import attention_varlen
    ctx = mp.get_context("spawn")
    q_ = ctx.Queue()
    port = 29060 + os.getpid() % 80
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q_)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q_.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    q, k, v, do, cu = _data()
    q, k, v = (t.clone().requires_grad_(True) for t in (q, k, v))
    o = attention_varlen(q, k, v, cu, True, 0.25)
    o.backward(do)
    n = q.shape[0] // 2
    for r, got in res.items():
        sl = slice(r * n, (r + 1) * n)
        for name, ref in (("o", o), ("dq", q.grad), ("dk", k.grad), ("dv", v.grad)):
            assert np.allclose(got[name], ref[sl].detach().numpy(), atol=1e-5), (r, name)
