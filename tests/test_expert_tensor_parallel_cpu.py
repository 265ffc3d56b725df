"""Expert tensor parallelism on gloo CPU ranks: ETP=2 alone and EP=2 x ETP=2,
forward and backward, against all experts unsharded on one rank."""

import os

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _check(ep: int, etp: int, T=48, H=64, F=96, E=4, k=2, seed=0) -> dict:
    from lumenrl_b200 import ops
    from lumenrl_b200.models.moe import grouped_linear
    from lumenrl_b200.parallel.expert_parallel import EPComm
    from lumenrl_b200.parallel.expert_tensor_parallel import etp_moe_forward, etp_shard_experts, make_ep_etp_groups
    W, r = dist.get_world_size(), dist.get_rank()
    etp_g, ep_g = make_ep_etp_groups(W, ep, etp)
    e_idx, j = r // etp, r % etp
    g = torch.Generator().manual_seed(seed)
    w13 = torch.randn(E, 2 * F, H, generator=g) / H ** 0.5
    w2 = torch.randn(E, H, F, generator=g) / F ** 0.5
    g.manual_seed(seed + 100 + r)
    h = torch.randn(T, H, generator=g)
    wts, ids = torch.softmax(torch.randn(T, E, generator=g), -1).topk(k, -1)
    dout = torch.randn(T, H, generator=g)
    # reference: every expert, unsharded, on this rank's tokens
    hr, wr = h.clone().requires_grad_(True), wts.clone().requires_grad_(True)
    W13, W2 = torch.nn.Parameter(w13.clone()), torch.nn.Parameter(w2.clone())
    flat = ids.reshape(-1)
    order = torch.argsort(flat, stable=True)
    offs = [0] + torch.cumsum(torch.bincount(flat, minlength=E), 0).tolist()
    ys = grouped_linear(ops.swiglu(grouped_linear(hr[order // k], W13, offs)), W2, offs)
    ref = torch.zeros_like(hr).index_add(0, order // k, ys * wr.reshape(-1)[order].unsqueeze(1))
    ref.backward(dout)
    # sharded: EP block of experts, ETP shard of their FFN
    El = E // ep
    b13, b2 = w13[e_idx * El:(e_idx + 1) * El], w2[e_idx * El:(e_idx + 1) * El]
    s13, s2 = etp_shard_experts(b13, b2, j, etp)
    L13, L2 = torch.nn.Parameter(s13), torch.nn.Parameter(s2)
    comm = EPComm(E, H, max_pairs=etp * T * k, capacity=W * T * k, group=ep_g, fused=False) if ep > 1 else None
    he, we = h.clone().requires_grad_(True), wts.clone().requires_grad_(True)
    out = etp_moe_forward(he, ids, we, L13, L2, etp_g, comm)
    out.backward(dout)
    g13, g2 = W13.grad.clone(), W2.grad.clone()
    dist.all_reduce(g13)
    dist.all_reduce(g2)
    r13, r2 = etp_shard_experts(g13[e_idx * El:(e_idx + 1) * El], g2[e_idx * El:(e_idx + 1) * El], j, etp)

    def rel(a, b):
        return ((a - b).abs().max() / b.abs().max().clamp(min=1e-12)).item()
    return {"out": rel(out, ref), "dh": rel(he.grad, hr.grad), "dw": rel(we.grad, wr.grad),
            "dw13": rel(L13.grad, r13), "dw2": rel(L2.grad, r2)}


def _worker(rank, world, port, ep, etp, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q.put((rank, _check(ep, etp)))
    except Exception as e:  # surfaced by the parent
        q.put((rank, {"error": repr(e)}))
    dist.destroy_process_group()


def _run(world, ep, etp, port):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, ep, etp, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, errs in res:
        assert "error" not in errs, (rank, errs)
        for key, v in errs.items():
            assert v < 1e-5, (rank, key, v)


def test_etp2_matches_unsharded_experts():
    _run(2, 1, 2, 29480 + os.getpid() % 100)


def test_ep2_x_etp2_matches_unsharded_experts():
    _run(4, 2, 2, 29600 + os.getpid() % 100)
