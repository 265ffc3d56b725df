"""Parameter-sharded training engine (ZeRO-3 / FSDP2-style full sharding;
reference: ``lumenrl/engine/training/fsdp_backend.py:251-366`` and
``lumenrl/engine/training/fsdp_engine.py:63-722``, where FSDP2
``fully_shard`` with ``reshard_after_forward`` keeps 1/W of every parameter
per rank).

``ActorEngine`` keeps the full bf16 weights resident on every GPU (they are
also the colocated rollout engine's weights) and shards only the fp32
optimizer state.  ``ShardedParamActorEngine`` shards the weights as well, for
models whose weights do not fit next to their activations: each rank holds
1/W of every *unit* (every decoder layer, and the outer unit of embedding,
final norm and LM head) in bf16, with its fp32 master, Adam moments and
gradient shard.

Per micro-batch:

* forward: the outer unit is gathered and kept for the micro-step; each
  decoder layer is gathered into a layer buffer just before it runs and its
  input is kept (no activations inside layers are saved);
* backward (the backward of one custom autograd function standing for the
  whole decoder stack): for each layer from the last, gather it again,
  recompute it with autograd, backpropagate the incoming gradient, and
  reduce-scatter the layer's fp32 weight gradients straight into this rank's
  gradient shard; the outer unit's gradients are reduce-scattered last.

Memory per GPU: 1/W of the weights and optimizer state, two layer-sized
weight buffers, one layer-sized fp32 gradient buffer and the layer inputs of
one micro-batch.  Every layer is recomputed (the forward runs twice), the
cost of full sharding.  The gathers and reduce-scatters are NCCL collectives
on the data-parallel group (gloo on CPU).

The optimizer step is local: AdamW on the shard with the gradient norm
all-reduced over the group; no parameter all-gather follows it, because the
next forward gathers layer by layer.  ``full_flat()`` assembles the whole
bf16 model (the ``Qwen3Model`` flat layout) when it is needed in one piece:
a weight push to rollout GPUs or an export.
"""

from __future__ import annotations

import math
import time
from typing import Optional

import torch
import torch.distributed as dist
from torch import Tensor

from lumenrl_b200 import ops
from lumenrl_b200.engine.training.actor import ActorEngine
from lumenrl_b200.engine.training.lr_scheduler import LRSchedule
from lumenrl_b200.models.config import ModelArgs
from lumenrl_b200.models.qwen3 import FlatLayout, Qwen3Model, embed, is_matrix, param_specs
from lumenrl_b200.parallel.dist import ParallelState

_ALIGN = 64   # elements: every tensor of a unit starts 128-byte aligned (bf16)


class _Unit:
    """Contiguous packing of some of the model's tensors, padded so it splits
    into W equal shards."""

    def __init__(self, names: list[str], layout: FlatLayout, world: int) -> None:
        self.names = names
        self.entries: dict[str, tuple[int, tuple[int, ...]]] = {}
        off = 0
        for n in names:
            shape = layout.entries[n][1]
            off = (off + _ALIGN - 1) // _ALIGN * _ALIGN
            self.entries[n] = (off, shape)
            off += math.prod(shape)
        q = world * _ALIGN
        self.numel = (off + q - 1) // q * q
        self.shard = self.numel // world
        self.shard_off = 0    # where this unit's shard starts in the rank's shard buffer


class _ShardAdamW:
    """AdamW on this rank's shards: fp32 master, moments and gradient; the
    gradient norm (for clipping and the non-finite skip) is summed over the
    data-parallel group."""

    def __init__(self, w16: Tensor, group, lr: float, betas, eps: float, weight_decay: float,
                 max_grad_norm: float) -> None:
        self.w16 = w16
        self.master = w16.float().clone()
        self.m = torch.zeros_like(self.master)
        self.v = torch.zeros_like(self.master)
        self.grad = torch.zeros_like(self.master)
        self.group = group
        self.lr, self.betas, self.eps, self.wd, self.max_grad_norm = lr, betas, eps, weight_decay, max_grad_norm
        self.step_count = 0
        self.last_timing: dict[str, float] = {}

    def step(self, lr: Optional[float] = None) -> dict:
        lr = self.lr if lr is None else lr
        t0 = time.perf_counter()
        ss = (self.grad.double() ** 2).sum().reshape(1)
        if dist.is_initialized():
            dist.all_reduce(ss, group=self.group)
        norm = float(ss.sqrt())
        clip = min(1.0, self.max_grad_norm / (norm + 1e-6)) if self.max_grad_norm and self.max_grad_norm > 0 else 1.0
        skipped = not math.isfinite(norm)
        if not skipped:
            self.step_count += 1
            b1, b2 = self.betas
            if self.master.is_cuda:
                from lumenrl_b200.ops.ext import ext
                ext().adamw_step(self.master, self.grad, self.m, self.v, self.w16, lr, b1, b2, self.eps, self.wd,
                                 self.step_count, clip)
            else:
                from lumenrl_b200.ops import reference as ref
                ref.adamw_reference(self.master, self.grad, self.m, self.v, lr, b1, b2, self.eps, self.wd,
                                    self.step_count, clip)
                self.w16.copy_(self.master.to(self.w16.dtype))
        self.grad.zero_()
        self.last_timing = {"opt_s": time.perf_counter() - t0}
        return {"grad_norm": norm, "skipped": float(skipped), "lr": lr, "clip_coef": clip}


class _ShardedStack(torch.autograd.Function):
    """The decoder stack of ``ShardedParamActorEngine`` as one autograd node:
    forward runs the layers without autograd (keeping each layer's input),
    backward recomputes and backpropagates them one gathered layer at a time."""

    @staticmethod
    def forward(ctx, eng, pb, anchor):
        x, pending, saved = eng._stack_forward(pb, keep_inputs=True)
        ctx.eng, ctx.pb, ctx.saved = eng, pb, saved
        return x, pending

    @staticmethod
    def backward(ctx, gx, gp):
        ctx.eng._stack_backward(ctx.pb, ctx.saved, gx, gp)
        ctx.saved = None
        return None, None, None


class ShardedParamActorEngine(ActorEngine):
    """``ActorEngine`` with the bf16 weights sharded over the data-parallel
    group (see the module docstring).  ``compute_log_probs`` and
    ``update_policy`` are the parent's; only the forward / backward and the
    optimizer differ."""

    def __init__(self, args: ModelArgs, state: ParallelState, *, lr: float = 1e-6, betas=(0.9, 0.999),
                 eps: float = 1e-8, weight_decay: float = 0.01, max_grad_norm: float = 1.0, seed: int = 0,
                 dtype: Optional[torch.dtype] = None, total_steps: int = 1000, warmup_steps: int = 0,
                 lr_style: str = "constant", min_lr_ratio: float = 0.0, gradient_checkpointing=None) -> None:
        # gradient_checkpointing is accepted for ActorEngine's signature: every
        # layer is recomputed here anyway
        if state.cp_size > 1:
            raise ValueError("parameter sharding is not combined with context parallelism")
        self.args, self.state, self.device = args, state, state.device
        if dtype is None:
            dtype = torch.bfloat16 if self.device.type == "cuda" else torch.float32
        self.dtype = dtype
        self.W, self.rank, self.group = state.world_size, state.rank, state.dp_group
        # the decoder code is Qwen3Model's; its tensors are views into gathered
        # unit buffers, rebound at every gather, so the model itself is built
        # on the meta device and never holds a full weight copy
        self.model = Qwen3Model(args, device="meta", dtype=dtype, requires_grad=True)
        self.model.inv_freq = ops.inv_freq_table(args.head_dim, args.rope_theta, args.rope_scaling, self.device)
        self.model.flat = None
        layout = self.model.layout
        names = layout.names()
        L = args.num_layers
        self.units = [_Unit([n for n in names if not n.startswith("layers.")], layout, self.W)]
        for i in range(L):
            self.units.append(_Unit([n for n in names if n.startswith(f"layers.{i}.")], layout, self.W))
        off = 0
        for u in self.units:
            u.shard_off = off
            off += u.shard
        self.w16 = torch.zeros(off, dtype=dtype, device=self.device)    # this rank's shards of every unit
        lmax = max(u.numel for u in self.units[1:])
        self.outer_buf = torch.zeros(self.units[0].numel, dtype=dtype, device=self.device)
        self.outer_grad = torch.zeros(self.units[0].numel, dtype=torch.float32, device=self.device)
        self.layer_bufs = [torch.zeros(lmax, dtype=dtype, device=self.device) for _ in range(2)]
        self.layer_grad = torch.zeros(lmax, dtype=torch.float32, device=self.device)
        self._init_shards(seed)
        self.opt = _ShardAdamW(self.w16, self.group, lr, betas, eps, weight_decay, max_grad_norm)
        self.sched = LRSchedule(lr, total_steps, warmup_steps, lr_style, min_lr_ratio)
        self.cp, self.cp_rank, self.cp_group = 1, 0, None
        self.comm = None
        self.trainable = True
        self.recompute_policy = None      # every layer is recomputed by construction
        self.model.gradient_checkpointing = False
        self._anchor = torch.zeros(1, device=self.device, requires_grad=True)
        self.comm_s = 0.0                 # host time in gathers / reduce-scatters (diagnostic)

    # ------------------------------------------------------------------ layout
    def _unit_of_layer(self, i: int) -> _Unit:
        return self.units[1 + i]

    def _shard(self, u: _Unit) -> Tensor:
        return self.w16[u.shard_off: u.shard_off + u.shard]

    @torch.no_grad()
    def _init_shards(self, seed: int) -> None:
        """The initialisation of ``Qwen3Model.init_weights`` (same per-tensor
        seeds), one unit at a time: every rank builds the unit and keeps its
        shard, so the sharded model equals an unsharded one with the seed."""
        std = self.args.init_std
        index = {n: i for i, n in enumerate(self.model.layout.names())}
        gen = torch.Generator(device=self.device)
        for u in self.units:
            full = torch.zeros(u.numel, dtype=self.dtype, device=self.device)
            for n, (o, shape) in u.entries.items():
                t = full[o: o + math.prod(shape)].view(shape)
                if is_matrix(n):
                    gen.manual_seed(seed * 7919 + index[n])
                    t.normal_(0.0, std, generator=gen)
                else:
                    t.fill_(1.0)
            self._shard(u).copy_(full[self.rank * u.shard:(self.rank + 1) * u.shard])

    # ------------------------------------------------------------------ collectives
    def _gather(self, u: _Unit, buf: Tensor) -> Tensor:
        t0 = time.perf_counter()
        out = buf[: u.numel]
        shard = self._shard(u)
        if self.W == 1:
            out.copy_(shard)
        elif out.is_cuda:
            dist.all_gather_into_tensor(out, shard, group=self.group)
        else:
            parts = [torch.empty_like(shard) for _ in range(self.W)]
            dist.all_gather(parts, shard, group=self.group)
            out.copy_(torch.cat(parts))
        self.comm_s += time.perf_counter() - t0
        return out

    def _reduce_scatter_grad(self, u: _Unit, gbuf: Tensor) -> None:
        """Sum the unit's full fp32 gradient over the group into this rank's
        gradient shard (accumulating over micro-batches)."""
        t0 = time.perf_counter()
        full = gbuf[: u.numel]
        dst = self.opt.grad[u.shard_off: u.shard_off + u.shard]
        if self.W == 1:
            dst += full
        elif full.is_cuda:
            part = torch.empty(u.shard, dtype=torch.float32, device=full.device)
            dist.reduce_scatter_tensor(part, full, group=self.group)
            dst += part
        else:
            dist.all_reduce(full, group=self.group)
            dst += full[self.rank * u.shard:(self.rank + 1) * u.shard]
        self.comm_s += time.perf_counter() - t0

    def _bind(self, u: _Unit, buf: Tensor, gbuf: Optional[Tensor]) -> None:
        """Point the model's tensors of unit ``u`` at the gathered ``buf``
        (leaf tensors whose weight gradients accumulate into ``gbuf``)."""
        for n, (o, shape) in u.entries.items():
            k = math.prod(shape)
            t = buf[o: o + k].view(shape).detach().requires_grad_(gbuf is not None)
            if gbuf is not None:
                t.main_grad = gbuf[o: o + k].view(shape)
            self.model._params[n] = t

    # ------------------------------------------------------------------ forward / backward
    def _stack_forward(self, pb, keep_inputs: bool):
        a, m = self.args, self.model
        x = embed(pb.input_ids, m.p("embed"))
        pending = None
        saved = []
        for i in range(a.num_layers):
            u = self._unit_of_layer(i)
            self._bind(u, self._gather(u, self.layer_bufs[i % 2]), None)
            if keep_inputs:
                saved.append((x, pending))
            x, pending = m._layer_fused(i, x, pending, pb.positions, pb.cu_seqlens, pb.max_seqlen)
        return x, pending, saved

    def _stack_backward(self, pb, saved, gx: Tensor, gp: Optional[Tensor]) -> None:
        m = self.model
        for i in reversed(range(self.args.num_layers)):
            u = self._unit_of_layer(i)
            self.layer_grad[: u.numel].zero_()
            self._bind(u, self._gather(u, self.layer_bufs[i % 2]), self.layer_grad)
            x_in, p_in = saved[i]
            x_in = x_in.detach().requires_grad_(True)
            p_in = p_in.detach().requires_grad_(True) if p_in is not None else None
            with torch.enable_grad():
                xo, po = m._layer_fused(i, x_in, p_in, pb.positions, pb.cu_seqlens, pb.max_seqlen)
            outs, grads = [xo], [gx]
            if gp is not None:
                outs.append(po)
                grads.append(gp)
            torch.autograd.backward(outs, grads)
            self._reduce_scatter_grad(u, self.layer_grad)
            gx = x_in.grad
            gp = p_in.grad if p_in is not None else None
        with torch.enable_grad():
            x0 = embed(pb.input_ids, m.p("embed"))
        x0.backward(gx)
        # the LM head and final norm finished their backward before this node
        self._reduce_scatter_grad(self.units[0], self.outer_grad)

    def _forward_scored(self, pb, temperature: float, want_entropy: bool):
        outer = self.units[0]
        training = torch.is_grad_enabled()
        if training:
            self.outer_grad.zero_()
        self._bind(outer, self._gather(outer, self.outer_buf), self.outer_grad if training else None)
        if training:
            x, pending = _ShardedStack.apply(self, pb, self._anchor)
        else:
            x, pending, _ = self._stack_forward(pb, keep_inputs=False)
        h, _ = ops.add_rmsnorm(x, pending, self.model.p("norm"), self.args.rms_norm_eps)
        hs = h.index_select(0, pb.score_index)
        return ops.token_logprob(hs, self.model.lm_head, pb.targets, temperature=temperature,
                                 want_entropy=want_entropy)

    def plan_recompute(self, tokens_per_micro: int, margin_bytes: int = 8 << 30) -> int:
        return self.args.num_layers

    # ------------------------------------------------------------------ whole model
    @torch.no_grad()
    def full_flat(self, numel: Optional[int] = None) -> Tensor:
        """The whole bf16 model in ``Qwen3Model``'s flat layout (a transient
        buffer, zero-padded to ``numel``): for weight pushes to rollout GPUs
        and exports.  Collective over the data-parallel group."""
        layout = FlatLayout(param_specs(self.args))
        flat = torch.zeros(max(layout.numel, numel or 0), dtype=self.dtype, device=self.device)
        tmp = torch.empty(max(u.numel for u in self.units), dtype=self.dtype, device=self.device)
        for u in self.units:
            full = self._gather(u, tmp)
            for n, (o, shape) in u.entries.items():
                layout.view(flat, n).copy_(full[o: o + math.prod(shape)].view(shape))
        return flat


def wants_param_sharding(config) -> bool:
    """``policy.training.fsdp_cfg.reshard_after_forward``: FSDP2's full
    sharding, i.e. this engine (where the trainer's weights are not also the
    colocated rollout's)."""
    fc = getattr(getattr(getattr(config, "policy", None), "training", None), "fsdp_cfg", None) or {}
    return bool(fc.get("reshard_after_forward", False)) if isinstance(fc, dict) else False
