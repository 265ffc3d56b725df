"""Expert parallelism on 2 CPU ranks (gloo all-to-all): dispatch -> grouped
experts -> combine, forward and backward, equals all experts on one rank."""

import os

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from lumenrl_b200.parallel.ep_check import ep_errors
    q.put((rank, ep_errors("cpu", torch.float32, fused=False)))
    dist.destroy_process_group()


def test_ep_moe_matches_local_experts_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29330 + os.getpid() % 150
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, errs in res:
        for k, v in errs.items():
            if k != "fused":
                assert v < 1e-5, (rank, k, v)
