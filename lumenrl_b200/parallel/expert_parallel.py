"""Expert parallelism for MoE layers (reference: Megatron's alltoall token
dispatcher with grouped GEMM, ``engine/training/megatron_native_engine.py:
284-353, 322-332, 403``; EP lockstep :1353-1370).

Rank d of ``W`` owns experts ``[d*E/W, (d+1)*E/W)``.  One MoE layer:

1. ``layout``: each rank sorts its (token, choice) pairs by expert and counts
   them; the ``[W, E]`` count table is exchanged (on GPUs by peer stores into
   every rank's table, ``ep_exchange_counts``; on CPU by an all-gather).  From
   the table every rank computes, on the device, where each of its pairs goes
   (owner rank, row in the owner's receive buffer, rows grouped by local
   expert then by source rank) and, for its own receive buffer, which rank and
   pair slot each row came from.
2. ``dispatch``: token rows are stored straight into the owners' receive
   buffers (``ep_scatter_rows``, plain NVLink stores, one flag per source).
3. the owner runs its experts on the received rows with the grouped tcgen05
   GEMM (offsets on the device);
4. ``combine``: each result row is stored back into the source rank's pair
   slot, and the source sums the k results of each token with the routing
   weights.

Backward mirrors it (combine's input gradient travels the dispatch route,
dispatch's the combine route).  Every rank must run the same sequence of MoE
layers.  Without NCCL (CPU, gloo) the transfers are ``all_to_all_single``,
which is also the reference the NVLink path is tested against.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist
from torch import Tensor

from lumenrl_b200 import ops

_COUNTS, _DISPATCH, _COMBINE, _COMBINE_BWD, _DISPATCH_BWD = 0, 1, 2, 3, 4


@dataclass
class Layout:
    order: Tensor        # [P] pair ids sorted by expert
    token_of: Tensor     # [P] token of each sorted pair
    dst_rank: Tensor     # [P] int32 owner rank of each sorted pair
    dst_row: Tensor      # [P] int32 row in the owner's receive buffer
    ret_rank: Tensor     # [cap] int32 source rank of each receive row
    ret_row: Tensor      # [cap] int32 source pair slot of each receive row (-1 = unused)
    offsets: Tensor      # [E_loc + 1] int32 local expert row offsets in the receive buffer
    send_splits: Optional[list] = None   # all-to-all path: rows per destination
    recv_splits: Optional[list] = None   # all-to-all path: rows per source
    recv_perm: Optional[Tensor] = None   # all-to-all path: receive order -> layout row


class EPComm:
    def __init__(self, num_experts: int, hidden: int, max_pairs: int, capacity: Optional[int] = None, group=None,
                 fused: Optional[bool] = None, wait_seconds: float = 10.0) -> None:
        self.group = group
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        if num_experts % self.world:
            raise ValueError("experts must divide by the EP size")
        self.E, self.E_loc, self.H = num_experts, num_experts // self.world, hidden
        self.max_pairs = max_pairs
        self.cap = capacity if capacity is not None else 2 * max_pairs
        cuda = torch.cuda.is_available() and dist.get_backend(group) == "nccl"
        self.fused = cuda if fused is None else (fused and cuda)
        self.wait_cycles = int(wait_seconds * 2.0e9)
        self.epoch = [0] * 16
        if self.fused:
            from lumenrl_b200.ops.ext import ext
            from lumenrl_b200.parallel.symm import SymmetricBuffer
            e = self._e = ext()
            W, r = self.world, self.rank
            self.recv = SymmetricBuffer(self.cap * hidden, torch.bfloat16, r, W, group)
            self.ret = SymmetricBuffer(max_pairs * hidden, torch.bfloat16, r, W, group)
            self.table = SymmetricBuffer(W * num_experts, torch.int32, r, W, group)
            self.sig = SymmetricBuffer(int(e.ep_flag_slots()), torch.int32, r, W, group)
            dev = self.recv.tensor.device
            self.status = torch.zeros(1, dtype=torch.int32, device=dev)
            self.counter = torch.zeros(1, dtype=torch.int32, device=dev)
            dist.barrier(group=group)

    def _next(self, slot: int) -> int:
        self.epoch[slot] += 1
        return self.epoch[slot]

    # ------------------------------------------------------------------ layout
    def layout(self, ids: Tensor) -> Layout:
        """``ids`` [T, k] expert ids -> routing of this layer."""
        W, E, El, r = self.world, self.E, self.E_loc, self.rank
        dev = ids.device
        k = ids.shape[1]
        flat = ids.reshape(-1)
        P = flat.numel()
        if P > self.max_pairs:
            raise ValueError(f"{P} pairs exceed max_pairs={self.max_pairs}")
        order = torch.argsort(flat, stable=True)
        counts = torch.bincount(flat, minlength=E).to(torch.int32)
        if self.fused:
            self._e.ep_exchange_counts(counts, self.table.ptrs, self.sig.ptrs, r, _COUNTS, self._next(_COUNTS),
                                       self.status, self.wait_cycles)
            table = self.table.tensor.view(W, E).clone()
        else:
            parts = [torch.empty_like(counts) for _ in range(W)]
            dist.all_gather(parts, counts, group=self.group)
            table = torch.stack(parts)
        tl = table.long()
        col = tl.sum(0)                                              # rows per expert, all sources
        colr = col.view(W, El)
        base = (torch.cumsum(colr, 1) - colr).reshape(E)             # expert start in its owner's buffer
        src_excl = torch.cumsum(tl, 0) - tl                          # [W, E] source start inside expert
        pair_excl = torch.cumsum(tl, 1) - tl                         # [W, E] sorted-pair base per source
        e_sorted = flat[order]
        dst_rank = (e_sorted // El).to(torch.int32)
        pos = torch.arange(P, device=dev) - pair_excl[r][e_sorted]
        dst_row = (base[e_sorted] + src_excl[r][e_sorted] + pos).to(torch.int32)
        # this rank's receive buffer: blocks (local expert, source)
        mine = tl[:, r * El:(r + 1) * El]                            # [W, El]
        blk = mine.t().reshape(-1)                                   # [(el, s)]
        blk_end = torch.cumsum(blk, 0)
        rows = torch.arange(self.cap, device=dev)
        b = torch.searchsorted(blk_end, rows, right=True).clamp(max=El * W - 1)
        el, s = b // W, b % W
        start = blk_end[b] - blk[b]
        ret_row = pair_excl[s, r * El + el] + (rows - start)
        valid = rows < blk_end[-1]
        ret_row = torch.where(valid, ret_row, torch.full_like(ret_row, -1)).to(torch.int32)
        offsets = torch.zeros(El + 1, dtype=torch.int32, device=dev)
        offsets[1:] = torch.cumsum(colr[r], 0)
        lay = Layout(order=order, token_of=order // k, dst_rank=dst_rank, dst_row=dst_row,
                     ret_rank=s.to(torch.int32), ret_row=ret_row, offsets=offsets)
        if not self.fused:
            per_dest = tl[r].view(W, El).sum(1)
            lay.send_splits = per_dest.tolist()
            lay.recv_splits = mine.sum(1).tolist()
            # all-to-all delivers source-major rows (each source's rows sorted by expert)
            lay.recv_perm = torch.cat([torch.cat([torch.arange(int(mine[si, ei]), device=dev)
                                                  + base[r * El + ei] + src_excl[si, r * El + ei]
                                                  for ei in range(El)]) for si in range(W)]) if W * El else rows[:0]
        return lay

    # ------------------------------------------------------------------ transfers
    def to_experts(self, rows: Tensor, lay: Layout, src_row: Optional[Tensor], slot: int) -> Tensor:
        """Pair rows (``rows[src_row[i]]`` or ``rows[i]``) -> receive buffers;
        returns this rank's receive rows [cap, H] (a copy)."""
        if self.fused:
            e = self._e
            ep = self._next(slot)
            e.ep_scatter_rows(rows.contiguous(), src_row, lay.dst_rank, lay.dst_row, self.recv.ptrs, self.cap,
                              self.sig.ptrs, self.rank, slot, ep, self.counter, self.status)
            e.ep_wait_all(self.sig.ptrs[self.rank], self.world, slot, ep, self.status, self.wait_cycles)
            return self.recv.tensor.view(self.cap, self.H).clone()
        send = rows if src_row is None else rows[src_row]
        got = send.new_empty(sum(lay.recv_splits), self.H)
        dist.all_to_all_single(got, send.contiguous(), lay.recv_splits, lay.send_splits, group=self.group)
        out = send.new_zeros(self.cap, self.H)
        out[lay.recv_perm] = got
        return out

    def to_sources(self, rows: Tensor, lay: Layout, P: int, slot: int) -> Tensor:
        """Receive-buffer rows [cap, H] -> the source ranks' pair slots;
        returns this rank's pair rows [P, H] in sorted-pair order (a copy)."""
        if self.fused:
            e = self._e
            ep = self._next(slot)
            e.ep_scatter_rows(rows.contiguous(), None, lay.ret_rank, lay.ret_row, self.ret.ptrs, self.max_pairs,
                              self.sig.ptrs, self.rank, slot, ep, self.counter, self.status)
            e.ep_wait_all(self.sig.ptrs[self.rank], self.world, slot, ep, self.status, self.wait_cycles)
            return self.ret.tensor.view(self.max_pairs, self.H)[:P].clone()
        send = rows[lay.recv_perm]
        got = rows.new_empty(P, self.H)
        dist.all_to_all_single(got, send.contiguous(), lay.send_splits, lay.recv_splits, group=self.group)
        return got

    def check(self) -> None:
        if self.fused:
            s = int(self.status.item())
            if s:
                from lumenrl_b200.parallel.symm import CommTimeout
                if s == 410:
                    raise RuntimeError("expert-parallel receive buffer overflow: raise the capacity")
                raise CommTimeout(f"expert-parallel exchange wait expired (code {s})")

    def close(self) -> None:
        if self.fused:
            torch.cuda.synchronize()
            for b in (self.recv, self.ret, self.table, self.sig):
                b.close()


class _Dispatch(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, comm, lay):
        ctx.comm, ctx.lay, ctx.T = comm, lay, h.shape[0]
        return comm.to_experts(h, lay, lay.token_of, _DISPATCH)

    @staticmethod
    def backward(ctx, g):
        comm, lay = ctx.comm, ctx.lay
        gp = comm.to_sources(g, lay, lay.order.numel(), _DISPATCH_BWD)
        dh = gp.new_zeros(ctx.T, gp.shape[1])
        dh.index_add_(0, lay.token_of, gp)
        return dh, None, None


class _Combine(torch.autograd.Function):
    @staticmethod
    def forward(ctx, y, w_sorted, comm, lay, T):
        ret = comm.to_sources(y, lay, lay.order.numel(), _COMBINE)
        out = ret.new_zeros(T, ret.shape[1])
        out.index_add_(0, lay.token_of, ret * w_sorted.to(ret.dtype).unsqueeze(1))
        ctx.save_for_backward(ret, w_sorted)
        ctx.comm, ctx.lay = comm, lay
        return out

    @staticmethod
    def backward(ctx, dout):
        ret, w_sorted = ctx.saved_tensors
        comm, lay = ctx.comm, ctx.lay
        g = dout[lay.token_of]
        dw = (g.float() * ret.float()).sum(-1)
        gy = comm.to_experts((g * w_sorted.to(g.dtype).unsqueeze(1)).contiguous(), lay, None, _COMBINE_BWD)
        return gy, dw, None, None, None


def ep_moe_forward(h: Tensor, ids: Tensor, weights: Tensor, w13_local: Tensor, w2_local: Tensor,
                   comm: EPComm) -> Tensor:
    """MoE expert part with experts spread over ``comm``'s ranks.  h [T, H],
    ids / weights [T, k] (routing of this rank's tokens), w13_local
    [E_loc, 2F, H], w2_local [E_loc, H, F] (this rank's experts)."""
    from lumenrl_b200.models.moe import _use_tc_grouped, grouped_linear, grouped_linear_device
    T = h.shape[0]
    lay = comm.layout(ids)
    w_sorted = weights.reshape(-1)[lay.order]
    x = _Dispatch.apply(h, comm, lay)
    if _use_tc_grouped(x, w13_local, w2_local):
        y = grouped_linear_device(ops.swiglu(grouped_linear_device(x, w13_local, lay.offsets)), w2_local,
                                  lay.offsets)
    else:
        offs = lay.offsets.tolist()
        y = grouped_linear(ops.swiglu(grouped_linear(x, w13_local, offs)), w2_local, offs)
    return _Combine.apply(y, w_sorted, comm, lay, T)
