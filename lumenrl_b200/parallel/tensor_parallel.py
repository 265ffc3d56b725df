"""Tensor parallelism with sequence parallelism (Megatron column/row-parallel
linears; reference ``engine/training/megatron_engine.py:203, 322-341,
431-451`` and ``megatron_native_engine.py:221, 384-406``).

Activations outside the linears are sharded by sequence (SP): rank r holds
tokens ``[r*Tl, (r+1)*Tl)``.  A column-parallel linear all-gathers its input
and multiplies by this rank's output rows; a row-parallel linear multiplies
this rank's input columns and reduce-scatters the result back to sequence
shards.  On B200 both collectives are fused into the GEMM
(``csrc/gemm/tp_gemm.cu``):

* ``ag_linear``: the GEMM's TMA producer reads each A tile straight from the
  rank that owns those rows (plain per-CTA TMA tile loads over NVLink),
  starting with its own rows while peers' ready flags arrive;
* ``linear_rs``: the GEMM epilogue stores each partial tile into the owning
  rank's receive slot, the owner sums the ``tp`` partials in fp32.

Backward uses the same two kernels the other way round (the input gradient of
a column-parallel linear is a GEMM + reduce-scatter, that of a row-parallel
linear an all-gather + GEMM); the weight gradients need the gathered input /
output gradient, gathered with NCCL.  With gloo (CPU) or ``fused=False``
every collective is the plain ``torch.distributed`` one, which is also the
reference the fused path is tested against.

Buffers are double-buffered and every call bumps a per-slot epoch, so a rank
never overwrites a shard or a receive slot that a peer may still read: it
only reuses a half after observing (in its previous call) that every peer
has moved past it.  All ranks must make the same sequence of calls.

``TPDecoderLayer`` shards one Qwen3/Llama decoder layer (attention heads and
MLP columns split across ``tp`` ranks) and runs it on sequence-sharded
activations.
"""

from __future__ import annotations

import math
from typing import Optional

import torch
import torch.distributed as dist
from torch import Tensor

from lumenrl_b200 import ops

_SLOTS = 16   # flag rows: 0/1 all-gather halves, 2/3 reduce-scatter halves


class TPComm:
    """Process-group handle plus, on CUDA with ``fused=True``, the symmetric
    buffers of the fused kernels.  ``max_ag`` / ``max_rs`` bound the elements
    of one all-gather shard and of one reduce-scatter output slot."""

    def __init__(self, group=None, fused: Optional[bool] = None, max_ag: int = 1 << 24, max_rs: int = 1 << 24,
                 wait_seconds: float = 10.0) -> None:
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        cuda = torch.cuda.is_available() and dist.get_backend(group) == "nccl"
        self.fused = cuda if fused is None else (fused and cuda)
        self.wait_cycles = int(wait_seconds * 2.0e9)
        if self.fused:
            from lumenrl_b200.ops.ext import ext
            from lumenrl_b200.parallel.symm import SymmetricBuffer
            self._e = ext()
            self.max_ag, self.max_rs = max_ag, max_rs
            self.ag = SymmetricBuffer(2 * max_ag, torch.bfloat16, self.rank, self.world, group)
            self.rs = SymmetricBuffer(2 * self.world * max_rs, torch.bfloat16, self.rank, self.world, group)
            self.sig = SymmetricBuffer(_SLOTS * 8, torch.int32, self.rank, self.world, group)
            dev = self.ag.tensor.device
            self.status = torch.zeros(1, dtype=torch.int32, device=dev)
            self.counter = torch.zeros(1, dtype=torch.int32, device=dev)
            self.ag_calls = 0
            self.rs_calls = 0
            dist.barrier(group=group)

    # ------------------------------------------------------------- reference collectives
    def all_gather(self, x: Tensor) -> Tensor:
        out = torch.empty((self.world * x.shape[0],) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
        dist.all_gather_into_tensor(out, x.contiguous(), group=self.group)
        return out

    def reduce_scatter(self, x: Tensor) -> Tensor:
        out = torch.empty((x.shape[0] // self.world,) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
        if x.is_cuda:
            dist.reduce_scatter_tensor(out, x.contiguous(), group=self.group)
        else:   # gloo has no reduce_scatter_tensor: all-reduce, keep this rank's rows
            y = x.contiguous().clone()
            dist.all_reduce(y, group=self.group)
            out.copy_(y.view(self.world, -1, *x.shape[1:])[self.rank])
        return out

    # ------------------------------------------------------------- fused collectives
    def ag_linear(self, x_local: Tensor, w: Tensor) -> Tensor:
        """AG(x_local) @ w^T -> [world * Tl, N]."""
        if (not self.fused or x_local.dtype != torch.bfloat16 or x_local.shape[0] % 128 or w.shape[0] % 8
                or x_local.shape[1] % 8):
            return self.all_gather(x_local) @ w.t()
        Tl, K = x_local.shape
        if Tl * K > self.max_ag:
            raise ValueError(f"all-gather shard of {Tl * K} elements exceeds the buffer ({self.max_ag})")
        self.ag_calls += 1
        par = self.ag_calls % 2          # double buffer: a peer may still read the other half
        epoch = (self.ag_calls + 1) // 2
        base = par * self.max_ag
        self.ag.tensor[base: base + Tl * K].view(Tl, K).copy_(x_local)
        e = self._e
        e.tp_publish(self.sig.ptrs, self.rank, par, epoch)
        ptrs = [p + base * 2 for p in self.ag.ptrs]
        return e.ag_gemm(ptrs, Tl, w.contiguous(), self.sig.ptrs, self.rank, par, epoch, self.status,
                         self.wait_cycles)

    def linear_rs(self, x: Tensor, w: Tensor) -> Tensor:
        """RS(x @ w^T) -> this rank's [T / world, N] rows."""
        T, N = x.shape[0], w.shape[0]
        if (not self.fused or x.dtype != torch.bfloat16 or T % (128 * self.world) or N % 8 or x.shape[1] % 8
                or (T // self.world) * N > self.max_rs):
            return self.reduce_scatter(x @ w.t())
        self.rs_calls += 1
        par = self.rs_calls % 2
        slot_elems = self.world * self.max_rs
        ptrs = [p + par * slot_elems * 2 for p in self.rs.ptrs]
        return self._e.gemm_rs(x.contiguous(), w.contiguous(), ptrs, self.sig.ptrs, self.counter, self.rank,
                               2 + par, (self.rs_calls + 1) // 2, self.status, self.wait_cycles)

    def check(self) -> None:
        if self.fused:
            s = int(self.status.item())
            if s:
                from lumenrl_b200.parallel.symm import CommTimeout
                raise CommTimeout(f"tensor-parallel collective wait expired (code {s})")

    def close(self) -> None:
        if self.fused:
            torch.cuda.synchronize()
            for b in (self.ag, self.rs, self.sig):
                b.close()


def _wgrad(w_handle: Tensor, dy: Tensor, x: Tensor) -> Optional[Tensor]:
    """dW = dy^T x, accumulated in fp32 into ``main_grad`` when present."""
    mg = getattr(w_handle, "main_grad", None)
    if mg is not None:
        if dy.is_cuda:
            torch.addmm(mg, dy.t(), x, out_dtype=torch.float32, out=mg)
        else:
            mg += dy.t().float() @ x.float()
        return None
    return (dy.t().float() @ x.float()).to(w_handle.dtype)


class _ColumnParallel(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x_local, w, w_handle, tp):
        ctx.save_for_backward(x_local, w)
        ctx.tp, ctx.w_handle = tp, w_handle
        return tp.ag_linear(x_local, w)

    @staticmethod
    def backward(ctx, dy):
        x_local, w = ctx.saved_tensors
        tp = ctx.tp
        dy = dy.contiguous()
        dx_local = tp.linear_rs(dy, w.t().contiguous())      # (dy @ W) reduce-scattered
        gw = _wgrad(ctx.w_handle, dy, tp.all_gather(x_local))
        return dx_local, None, gw, None


class _RowParallel(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, w_handle, tp):
        ctx.save_for_backward(x, w)
        ctx.tp, ctx.w_handle = tp, w_handle
        return tp.linear_rs(x.contiguous(), w)

    @staticmethod
    def backward(ctx, dy_local):
        x, w = ctx.saved_tensors
        tp = ctx.tp
        dy_local = dy_local.contiguous()
        dx = tp.ag_linear(dy_local, w.t().contiguous())     # AG(dy) @ W
        gw = _wgrad(ctx.w_handle, tp.all_gather(dy_local), x)
        return dx, None, gw, None


def column_parallel(x_local: Tensor, w: Tensor, tp: TPComm) -> Tensor:
    """[Tl, K] sequence shard -> [T, N_local] (all-gather fused into the GEMM)."""
    if not torch.is_grad_enabled():
        return tp.ag_linear(x_local, w)
    return _ColumnParallel.apply(x_local, w.detach(), w, tp)


def row_parallel(x: Tensor, w: Tensor, tp: TPComm) -> Tensor:
    """[T, K_local] -> [Tl, N] sequence shard (reduce-scatter fused into the GEMM)."""
    if not torch.is_grad_enabled():
        return tp.linear_rs(x.contiguous(), w)
    return _RowParallel.apply(x, w.detach(), w, tp)


# ---------------------------------------------------------------------- sharding
def shard_qkv(wqkv: Tensor, nh: int, nkv: int, hd: int, rank: int, world: int) -> Tensor:
    q, k, v = wqkv.split([nh * hd, nkv * hd, nkv * hd], 0)
    qh, kh = nh // world, nkv // world
    return torch.cat([q[rank * qh * hd: (rank + 1) * qh * hd], k[rank * kh * hd: (rank + 1) * kh * hd],
                      v[rank * kh * hd: (rank + 1) * kh * hd]], 0)


def shard_rows(w: Tensor, rank: int, world: int) -> Tensor:
    n = w.shape[0] // world
    return w[rank * n: (rank + 1) * n]


def shard_cols(w: Tensor, rank: int, world: int) -> Tensor:
    n = w.shape[1] // world
    return w[:, rank * n: (rank + 1) * n]


def shard_gate_up(w13: Tensor, rank: int, world: int) -> Tensor:
    g, u = w13.chunk(2, 0)
    return torch.cat([shard_rows(g, rank, world), shard_rows(u, rank, world)], 0)


class TPDecoderLayer(torch.nn.Module):
    """One dense Qwen3/Llama decoder layer with its heads and MLP columns split
    over the ``tp`` ranks of ``comm``; activations are sequence shards.  The
    norm weights are replicated: their gradients are partial sums over this
    rank's tokens and must be all-reduced over the TP group (as in Megatron
    with sequence parallelism)."""

    def __init__(self, args, full_params: dict, comm: TPComm, inv_freq: Tensor) -> None:
        super().__init__()
        W, r = comm.world, comm.rank
        if args.num_heads % W or args.num_kv_heads % W or args.intermediate_size % W:
            raise ValueError("heads, kv heads and intermediate size must divide by the TP size")
        self.args, self.comm = args, comm
        self.nh, self.nkv = args.num_heads // W, args.num_kv_heads // W

        def P(t):
            return torch.nn.Parameter(t.detach().clone().contiguous())
        self.ln1 = P(full_params["ln1"])
        self.ln2 = P(full_params["ln2"])
        self.wqkv = P(shard_qkv(full_params["wqkv"], args.num_heads, args.num_kv_heads, args.head_dim, r, W))
        self.wo = P(shard_cols(full_params["wo"], r, W))
        self.w13 = P(shard_gate_up(full_params["w13"], r, W))
        self.w2 = P(shard_cols(full_params["w2"], r, W))
        self.q_norm = P(full_params["q_norm"]) if "q_norm" in full_params else None
        self.k_norm = P(full_params["k_norm"]) if "k_norm" in full_params else None
        self.register_buffer("inv_freq", inv_freq, persistent=False)

    def forward(self, x_local: Tensor, positions: Tensor, cu: Tensor, max_len: int) -> Tensor:
        a, tp = self.args, self.comm
        h = ops.rmsnorm(x_local, self.ln1, a.rms_norm_eps)
        qkv = column_parallel(h, self.wqkv, tp)
        q, k, v = ops.qk_norm_rope(qkv, self.q_norm, self.k_norm, positions, self.inv_freq, self.nh, self.nkv,
                                   a.head_dim, a.rms_norm_eps)
        o = ops.attention_varlen(q, k, v, cu, max_len, causal=True, scale=1.0 / math.sqrt(a.head_dim))
        x_local = x_local + row_parallel(o.reshape(o.shape[0], -1), self.wo, tp)
        h = ops.rmsnorm(x_local, self.ln2, a.rms_norm_eps)
        y = row_parallel(ops.swiglu(column_parallel(h, self.w13, tp)), self.w2, tp)
        return x_local + y
