"""Equivalence check of the expert-parallel MoE part against all experts on
one rank (run by every rank of a process group; used by the gloo CPU test and
the 2-GPU test of the NVLink dispatch / combine).  Errors are relative:
max |ep - ref| / max |ref|."""

from __future__ import annotations

import torch
import torch.distributed as dist


def ep_errors(device: str, dtype: torch.dtype, fused: bool, T: int = 96, H: int = 128, F: int = 128, E: int = 8,
              k: int = 2, seed: int = 0) -> dict:
    from lumenrl_b200 import ops
    from lumenrl_b200.models.moe import grouped_linear
    from lumenrl_b200.parallel.expert_parallel import EPComm, ep_moe_forward
    W, r = dist.get_world_size(), dist.get_rank()
    g = torch.Generator(device=device).manual_seed(seed)
    w13 = (torch.randn(E, 2 * F, H, device=device, generator=g) / H ** 0.5).to(dtype)
    w2 = (torch.randn(E, H, F, device=device, generator=g) / F ** 0.5).to(dtype)
    # every rank has its own tokens and routing
    g.manual_seed(seed + 100 + r)
    h = torch.randn(T, H, device=device, generator=g).to(dtype)
    logits = torch.randn(T, E, device=device, generator=g)
    wts, ids = torch.softmax(logits, -1).topk(k, -1)
    dout = torch.randn(T, H, device=device, generator=g).to(dtype)
    # reference: all experts here
    hr = h.clone().requires_grad_(True)
    wr = wts.clone().requires_grad_(True)
    W13, W2 = torch.nn.Parameter(w13.clone()), torch.nn.Parameter(w2.clone())
    flat = ids.reshape(-1)
    order = torch.argsort(flat, stable=True)
    offs = [0] + torch.cumsum(torch.bincount(flat, minlength=E), 0).tolist()
    xs = hr[order // k]
    ys = grouped_linear(ops.swiglu(grouped_linear(xs, W13, offs)), W2, offs)
    ref = torch.zeros_like(hr).index_add(0, order // k, ys * wr.reshape(-1)[order].to(ys.dtype).unsqueeze(1))
    ref.backward(dout)
    # expert parallel
    El = E // W
    comm = EPComm(E, H, max_pairs=T * k, capacity=W * T * k, fused=fused)
    he = h.clone().requires_grad_(True)
    we = wts.clone().requires_grad_(True)
    L13 = torch.nn.Parameter(w13[r * El:(r + 1) * El].clone())
    L2 = torch.nn.Parameter(w2[r * El:(r + 1) * El].clone())
    out = ep_moe_forward(he, ids, we, L13, L2, comm)
    out.backward(dout)
    if device == "cuda":
        torch.cuda.synchronize()
    comm.check()
    comm.close()

    def rel(a, b):
        return ((a.float() - b.float()).abs().max() / b.float().abs().max().clamp(min=1e-12)).item()
    # expert weight grads: sum the per-rank reference grads (each rank's tokens) over ranks
    g13, g2 = W13.grad.float().clone(), W2.grad.float().clone()
    dist.all_reduce(g13)
    dist.all_reduce(g2)
    return {"out": rel(out, ref), "dh": rel(he.grad, hr.grad), "dw": rel(we.grad, wr.grad),
            "dw13": rel(L13.grad, g13[r * El:(r + 1) * El]), "dw2": rel(L2.grad, g2[r * El:(r + 1) * El]),
            "fused": comm.fused}
