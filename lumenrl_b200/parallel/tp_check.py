"""Equivalence check of a tensor+sequence-parallel decoder layer against the
unsharded layer, run by every rank of a process group (used by the gloo CPU
test and the 2-GPU test of the fused NVLink kernels).  Errors are relative:
max |tp - full| / max |full|.

Each rank builds the same full layer, runs it on the whole sequence, then
runs its TP shard on its sequence slice and returns the largest differences
of the output, the input gradient and every weight gradient (replicated norm
weights' gradients are summed over the TP ranks first, as SP requires).
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def tp_layer_errors(device: str, dtype: torch.dtype, fused: bool, T: int = 512, seed: int = 0) -> dict:
    from lumenrl_b200.models.config import tiny_qwen3
    from lumenrl_b200.models.qwen3 import Qwen3Model
    from lumenrl_b200.parallel.tensor_parallel import (TPComm, TPDecoderLayer, shard_cols, shard_gate_up,
                                                       shard_qkv)
    args = tiny_qwen3(layers=1)
    m = Qwen3Model(args, device=device, dtype=dtype, requires_grad=True)
    m.init_weights(seed, std=0.05)
    comm = TPComm(fused=fused)
    W, r = comm.world, comm.rank
    g = torch.Generator(device=device).manual_seed(seed + 1)
    x = torch.randn(T, args.hidden_size, device=device, generator=g).to(dtype)
    dy = torch.randn(T, args.hidden_size, device=device, generator=g).to(dtype)
    lens = [T // 2 - 32, T // 2 + 32]
    cu = torch.tensor([0, lens[0], T], dtype=torch.int32, device=device)
    pos = torch.cat([torch.arange(n, device=device) for n in lens])
    # full layer on the whole sequence
    xf = x.clone().requires_grad_(True)
    yf = m._layer(0, xf, pos, cu, max(lens))
    (yf.float() * dy.float()).sum().backward()
    full = {k.split(".", 2)[2]: p for k, p in m.named_flat_params() if k.startswith("layers.0.")}
    grads = {k: p.grad.float() for k, p in full.items()}
    # TP layer on this rank's sequence slice
    layer = TPDecoderLayer(args, full, comm, m.inv_freq)
    Tl = T // W
    xl = x[r * Tl: (r + 1) * Tl].clone().requires_grad_(True)
    yl = layer(xl, pos, cu, max(lens))
    (yl.float() * dy[r * Tl: (r + 1) * Tl].float()).sum().backward()
    if device == "cuda":
        torch.cuda.synchronize()
    comm.check()

    def rel(a, b):
        return ((a.float() - b.float()).abs().max() / b.float().abs().max().clamp(min=1e-12)).item()

    errs = {"y": rel(yl, yf[r * Tl: (r + 1) * Tl]), "dx": rel(xl.grad, xf.grad[r * Tl: (r + 1) * Tl])}
    expect = {"wqkv": shard_qkv(grads["wqkv"], args.num_heads, args.num_kv_heads, args.head_dim, r, W),
              "wo": shard_cols(grads["wo"], r, W), "w13": shard_gate_up(grads["w13"], r, W),
              "w2": shard_cols(grads["w2"], r, W)}
    for name, ref in expect.items():
        errs[name] = rel(getattr(layer, name).grad, ref)
    for name in ("ln1", "ln2", "q_norm", "k_norm"):
        gsum = getattr(layer, name).grad.float().clone()
        dist.all_reduce(gsum)
        errs[name] = rel(gsum, grads[name])
    errs["fused"] = comm.fused
    comm.close()
    return errs
