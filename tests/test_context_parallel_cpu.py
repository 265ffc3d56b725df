"""Context parallelism on 2 and 3 CPU ranks (gloo): zigzag ring attention's
output and q/k/v gradients equal full causal attention (fp32), GQA included;
the sequence gather is differentiable."""

import math
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _data(S, H=4, Hk=2, D=16, seed=0):
    g = torch.Generator().manual_seed(seed)
    q, k, v = (torch.randn(1, h, S, D, generator=g) for h in (H, Hk, Hk))
    do = torch.randn(1, H, S, D, generator=g)
    return q, k, v, do


def _full(q, k, v, do):
    q, k, v = (t.clone().requires_grad_(True) for t in (q, k, v))
    H = q.shape[1]
    ke, ve = k.repeat_interleave(H // k.shape[1], 1), v.repeat_interleave(H // v.shape[1], 1)
    s = (q @ ke.transpose(-1, -2)) / math.sqrt(q.shape[-1])
    S = s.shape[-1]
    s = s.masked_fill(torch.ones(S, S, dtype=torch.bool).triu(1), float("-inf"))
    o = torch.softmax(s, -1) @ ve
    o.backward(do)
    return o.detach(), q.grad, k.grad, v.grad


def _worker(rank, world, port, S, q_out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from lumenrl_b200.parallel.context_parallel import gather_seq, ring_attention, zigzag_indices
    q, k, v, do = _data(S)
    idx = zigzag_indices(S, world, rank)
    ql, kl, vl = (t[:, :, idx].clone().requires_grad_(True) for t in (q, k, v))
    o = ring_attention(ql, kl, vl)
    o.backward(do[:, :, idx])
    # the gathered sequence is differentiable: sum of a weighted full tensor
    x = torch.arange(S, dtype=torch.float32)[idx].clone().requires_grad_(True)
    full = gather_seq(x.unsqueeze(-1), S)
    (full.squeeze(-1) * torch.arange(S, dtype=torch.float32)).sum().backward()
    res = {n: t.detach().numpy().copy() for n, t in
           (("o", o), ("dq", ql.grad), ("dk", kl.grad), ("dv", vl.grad), ("full", full), ("dx", x.grad))}
    q_out.put((rank, idx.numpy(), res))
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_ring_attention_matches_full(world):
    S = 24
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29400 + 10 * world + os.getpid() % 90
    procs = [ctx.Process(target=_worker, args=(r, world, port, S, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    o, dq, dk, dv = _full(*_data(S))
    for rank, idx, r in res:
        idx = torch.from_numpy(idx)
        for name, ref in (("o", o), ("dq", dq), ("dk", dk), ("dv", dv)):
            got = torch.from_numpy(r[name])
            assert torch.allclose(got, ref[:, :, idx], atol=1e-5), (rank, name, (got - ref[:, :, idx]).abs().max())
        assert np.allclose(r["full"].squeeze(-1), np.arange(S))
        # d/dx of sum_ranks(sum_t t * full_t) = world * position
        assert np.allclose(r["dx"], world * idx.numpy())
