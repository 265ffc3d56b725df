"""Expert tensor parallelism (ETP): every expert's FFN split over ``t`` ranks.

Reference: Megatron's expert-tensor-parallel size
(``engine/training/megatron_engine.py:216-218, 433-451``): the experts' fc1
is column-parallel and fc2 row-parallel inside an ETP group, tokens are
gathered over the group before the experts and the partial outputs are
reduce-scattered after them.

Layout.  ETP rank ``j`` of ``t`` holds rows ``[j F/t, (j+1) F/t)`` of the
gate and of the up projection (``w13`` keeps its [gate; up] stacking, so the
SwiGLU of a shard needs no communication) and the matching columns of
``w2``.  Each rank keeps its own (sequence-parallel) tokens; one MoE layer:

1. all-gather the group's tokens, routing ids and routing weights;
2. run the experts on the gathered tokens with this rank's FFN shards --
   locally (``ep_comm=None``) or, composed with expert parallelism, through
   ``ep_moe_forward`` inside the EP group of ranks that hold the same ETP
   shard of other experts;
3. reduce-scatter the partial outputs back to the token owners.

Backward: the gather's gradient is a reduce-scatter and the scatter's an
all-gather.  The collectives are NCCL ``all_gather_into_tensor`` /
``reduce_scatter_tensor`` (gloo: all-gather / all-reduce + slice); unlike the
dense TP path (``csrc/gemm/tp_gemm.cu``) they are not fused into the grouped
GEMM.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist
from torch import Tensor


def etp_shard_experts(w13: Tensor, w2: Tensor, rank: int, size: int) -> tuple[Tensor, Tensor]:
    """(w13 [E, 2F, H], w2 [E, H, F]) -> this ETP rank's ([E, 2F/t, H], [E, H, F/t])."""
    F = w2.shape[2]
    if F % size:
        raise ValueError(f"expert FFN width {F} is not divisible by the ETP size {size}")
    f = F // size
    a, b = rank * f, (rank + 1) * f
    return torch.cat([w13[:, a:b], w13[:, F + a:F + b]], 1).contiguous(), w2[:, :, a:b].contiguous()


def make_ep_etp_groups(world: int, ep: int, etp: int):
    """Rank ``e * etp + j`` is ETP rank ``j`` of EP rank ``e``.  Returns this
    rank's (etp_group, ep_group); every rank creates every group."""
    if ep * etp != world:
        raise ValueError(f"ep {ep} x etp {etp} != world {world}")
    me = dist.get_rank()
    etp_g = ep_g = None
    for e in range(ep):
        ranks = [e * etp + j for j in range(etp)]
        g = dist.new_group(ranks)
        if me in ranks:
            etp_g = g
    for j in range(etp):
        ranks = [e * etp + j for e in range(ep)]
        g = dist.new_group(ranks)
        if me in ranks:
            ep_g = g
    return etp_g, ep_g


def _nccl(group) -> bool:
    return dist.get_backend(group) == "nccl"


def _gather_rows(x: Tensor, group) -> Tensor:
    t = dist.get_world_size(group)
    out = x.new_empty(t * x.shape[0], *x.shape[1:])
    if _nccl(group):
        dist.all_gather_into_tensor(out, x.contiguous(), group=group)
    else:
        dist.all_gather(list(out.chunk(t)), x.contiguous(), group=group)
    return out


def _scatter_rows(x: Tensor, group) -> Tensor:
    """Sum over the group, keep this rank's block of rows."""
    t, r = dist.get_world_size(group), dist.get_rank(group)
    n = x.shape[0] // t
    if _nccl(group):
        out = x.new_empty(n, *x.shape[1:])
        dist.reduce_scatter_tensor(out, x.contiguous(), group=group)
        return out
    y = x.contiguous().clone()
    dist.all_reduce(y, group=group)
    return y[r * n:(r + 1) * n].contiguous()


class _GatherRows(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return _gather_rows(x, group)

    @staticmethod
    def backward(ctx, g):
        return _scatter_rows(g, ctx.group), None


class _ScatterRows(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return _scatter_rows(x, group)

    @staticmethod
    def backward(ctx, g):
        return _gather_rows(g, ctx.group), None


def _local_experts(h: Tensor, ids: Tensor, weights: Tensor, w13: Tensor, w2: Tensor) -> Tensor:
    from lumenrl_b200 import ops
    from lumenrl_b200.models.moe import _use_tc_grouped, grouped_linear, grouped_linear_device
    T, k = ids.shape
    E = w13.shape[0]
    flat = ids.reshape(-1)
    order = torch.argsort(flat, stable=True)
    counts = torch.bincount(flat, minlength=E)
    token_of = order // k
    xs = h[token_of]
    if _use_tc_grouped(h, w13, w2):
        offs = torch.zeros(E + 1, dtype=torch.int32, device=h.device)
        offs[1:] = torch.cumsum(counts, 0)
        ys = grouped_linear_device(ops.swiglu(grouped_linear_device(xs, w13, offs)), w2, offs)
    else:
        offsets = [0] + torch.cumsum(counts, 0).tolist()
        ys = grouped_linear(ops.swiglu(grouped_linear(xs, w13, offsets)), w2, offsets)
    wt = weights.reshape(-1)[order].to(ys.dtype).unsqueeze(-1)
    return torch.zeros_like(h).index_add(0, token_of, ys * wt)


def etp_moe_forward(h: Tensor, ids: Tensor, weights: Tensor, w13_shard: Tensor, w2_shard: Tensor, etp_group,
                    ep_comm: Optional[object] = None) -> Tensor:
    """Expert part of a MoE layer under ETP (and optionally EP).
    h [T, H] this rank's tokens (every rank of the ETP group has the same T);
    ids / weights [T, k] their routing; w13_shard / w2_shard this rank's FFN
    shards of its experts (all experts, or the EP-local ones with
    ``ep_comm``)."""
    hg = _GatherRows.apply(h, etp_group)
    idg = _gather_rows(ids, etp_group)
    wg = _GatherRows.apply(weights, etp_group)
    if ep_comm is None:
        part = _local_experts(hg, idg, wg, w13_shard, w2_shard)
    else:
        from lumenrl_b200.parallel.expert_parallel import ep_moe_forward
        part = ep_moe_forward(hg, idg, wg, w13_shard, w2_shard, ep_comm)
    return _ScatterRows.apply(part, etp_group)
