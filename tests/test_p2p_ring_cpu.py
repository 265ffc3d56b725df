"""Hidden-state ring over torch.distributed send/recv (gloo, 2 CPU ranks):
the producer's batches arrive in order and intact at the consumer."""

import os

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from lumenrl_b200.transfer.p2p_ring import HiddenStateRing
    ring = HiddenStateRing(producer=0, consumer=1, slot_bytes=4 * 64 * 12, nslots=2)
    ok = True
    for i in range(5):
        x = torch.full((64, 12), float(i)) + torch.arange(12.0)
        if rank == 0:
            ring.put(x)
        else:
            y = ring.get((64, 12), torch.float32)
            ok &= torch.equal(x, y)
            ring.release()
    q.put((rank, ok, ring.backend))
    dist.barrier()
    dist.destroy_process_group()


def test_ring_over_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 150
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict((r, (ok, b)) for r, ok, b in (q.get(timeout=120) for _ in procs))
    for p in procs:
        p.join(timeout=60)
    assert res[1][0] and res[1][1] == "pg"
