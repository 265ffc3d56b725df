"""Tensor + sequence parallelism on 2 CPU ranks (gloo): the sharded decoder
layer's output, input gradient and weight gradients equal the unsharded
layer's (fp32)."""

import os

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from lumenrl_b200.parallel.tp_check import tp_layer_errors
    q.put((rank, tp_layer_errors("cpu", torch.float32, fused=False, T=128)))
    dist.destroy_process_group()


def test_tp_layer_matches_unsharded_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29650 + os.getpid() % 150
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, errs in res:
        for k, v in errs.items():
            if k == "fused":
                continue
            assert v < 1e-5, (rank, k, v)
