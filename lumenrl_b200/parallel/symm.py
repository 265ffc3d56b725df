"""Symmetric device buffers over CUDA IPC and the fused NVLink optimizer step.

``SymmetricBuffer(numel, dtype, group)`` allocates the same-sized buffer on
every rank (outside the caching allocator), exchanges CUDA IPC handles over
the process group and maps every peer's copy, so the fused kernels in
``csrc/comm/symm.cu`` can load from and store to any rank's buffer directly
over NVLink / NVSwitch.

``NVLinkOptimizerComm`` owns the three symmetric buffers of a sharded
trainer (flat bf16 weights, flat fp32 gradients, signal flags) and runs the
optimizer step as two fused kernels:

1. ``rs_norm``: cross-rank barrier, reduce-scatter of the fp32 gradients by
   peer loads into this rank's shard, and its sum of squares published to
   every rank;
2. ``adamw_ag``: barrier, global-norm clip (non-finite -> skip), AdamW on the
   fp32 master shard, and the bf16 result stored into EVERY rank's resident
   weight buffer -- the parameter all-gather and the trainer -> rollout
   weight sync in the same pass -- then a completion barrier.

With ``nvls`` (opt-in: ``nvls=True`` or ``LRL_NVLS=1``, used when the GPUs
support NVLink SHARP multicast) the
weight and gradient buffers come from PyTorch's symmetric memory, which also
maps them into one NVLS multicast object; the kernels then use
``multimem.ld_reduce`` (the gradient sum of an element over all GPUs, reduced
in the NVSwitch) and ``multimem.st`` (one store into every GPU's weights), so
each byte crosses a GPU's NVLink ports once.

Waits are bounded in the kernels; ``check()`` raises ``CommTimeout`` when a
kernel recorded an expired wait (a dead or stalled rank).
"""

from __future__ import annotations

import os
from typing import Optional

import torch
import torch.distributed as dist

from lumenrl_b200.ops.ext import ext


class CommTimeout(RuntimeError):
    pass


class SymmetricBuffer:
    def __init__(self, numel: int, dtype: torch.dtype, rank: int, world: int, group=None) -> None:
        self.numel, self.dtype, self.rank, self.world = numel, dtype, rank, world
        nbytes = numel * torch.empty(0, dtype=dtype).element_size()
        words = ext().symm_malloc(nbytes)
        self.local_ptr = int(words[0])
        handle = [int(w) for w in words[1:]]
        handles: list = [None] * world
        dist.all_gather_object(handles, handle, group=group)
        self.ptrs: list[int] = []
        self._opened: list[int] = []
        for r, h in enumerate(handles):
            if r == rank:
                self.ptrs.append(self.local_ptr)
            else:
                p = int(ext().symm_open(h))
                ext().bounds_register(p, nbytes)   # extent for the bounds-checked comm kernels
                self.ptrs.append(p)
                self._opened.append(p)
        self.tensor = ext().symm_tensor(self.local_ptr, numel, dtype)

    def close(self) -> None:
        for p in self._opened:
            ext().symm_close(p)
        self._opened = []
        if self.local_ptr:
            ext().symm_free(self.local_ptr)
            self.local_ptr = 0


class MulticastBuffer:
    """Same-sized buffer on every rank from PyTorch's symmetric memory (cuMem
    allocations mapped into every peer) plus its NVLS multicast address
    ``mc`` (0 when the GPUs have no multicast support)."""

    def __init__(self, numel: int, dtype: torch.dtype, group=None) -> None:
        import torch.distributed._symmetric_memory as symm
        g = group if group is not None else dist.group.WORLD
        try:
            symm.enable_symm_mem_for_group(g.group_name)
        except Exception:
            pass
        dev = torch.device("cuda", torch.cuda.current_device())
        self.tensor = symm.empty(numel, dtype=dtype, device=dev)
        self.tensor.zero_()
        self.handle = symm.rendezvous(self.tensor, g.group_name)
        self.ptrs = [int(p) for p in self.handle.buffer_ptrs]
        self.mc = int(self.handle.multicast_ptr)
        nbytes = numel * self.tensor.element_size()
        for p in self.ptrs:
            ext().bounds_register(p, nbytes)   # extents for the bounds-checked comm kernels

    def close(self) -> None:
        if self.handle is not None:
            for p in self.ptrs:
                ext().bounds_unregister(p)
        self.handle = None


def nvls_supported() -> bool:
    try:
        import torch.distributed._symmetric_memory as symm
        from torch._C._distributed_c10d import _SymmetricMemory
        return bool(_SymmetricMemory.has_multicast_support(torch._C._autograd.DeviceType.CUDA,
                                                           torch.cuda.current_device()))
    except Exception:
        return False


class NVLinkOptimizerComm:
    """Fused reduce-scatter / AdamW / all-gather over NVLink peer memory, or
    over NVLS multicast (``nvls``: True, False, or None = ``LRL_NVLS`` == "1";
    either way only when the GPUs support it)."""

    def __init__(self, numel: int, rank: int, world: int, weight_dtype=torch.bfloat16, group=None,
                 wait_seconds: float = 10.0, nvls: Optional[bool] = None) -> None:
        self.rank, self.world, self.group = rank, world, group
        # in-kernel spin bound, in SM clock cycles at boost clock
        self.wait_cycles = int(wait_seconds * 2.0e9)
        if nvls is None:   # LRL_NVLS=1 opts in; the unicast peer path is the default
            nvls = os.environ.get("LRL_NVLS", "0") == "1"
        use_mc = bool(nvls) and nvls_supported()
        self.nvls = False
        if use_mc:
            self.weights = MulticastBuffer(numel, weight_dtype, group)
            self.grads = MulticastBuffer(numel, torch.float32, group)
            self.nvls = self.weights.mc != 0 and self.grads.mc != 0
            if not self.nvls:
                self.weights.close()
                self.grads.close()
        if not self.nvls:
            self.weights = SymmetricBuffer(numel, weight_dtype, rank, world, group)
            self.grads = SymmetricBuffer(numel, torch.float32, rank, world, group)
        self.signals = SymmetricBuffer(int(ext().symm_signal_words()), torch.int32, rank, world, group)
        dev = self.weights.tensor.device
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        self.norm = torch.zeros(1, dtype=torch.float32, device=dev)
        self.epoch = 0
        self.last_timing: dict[str, float] = {}
        self._rendezvous = torch.zeros(1, dtype=torch.int32, device=dev)
        dist.barrier(group=group)

    def fused_step(self, shard_lo: int, shard_n: int, master, grad_shard, m, v, lr: float, betas, eps: float,
                   wd: float, step: int, max_norm: float, rendezvous: bool = True) -> tuple[float, bool]:
        self.epoch += 1
        e = ext()
        # stream-ordered rendezvous (4 bytes over NCCL, control plane only): ranks
        # whose backward finished at different times meet here, so the in-kernel
        # flag barriers below only order memory and never wait long
        if rendezvous:
            dist.all_reduce(self._rendezvous, group=self.group)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        ev[0].record()
        if self.nvls:
            e.rs_norm_mc(self.grads.mc, self.signals.ptrs, self.rank, shard_lo, shard_n, grad_shard, self.epoch,
                         self.status, self.wait_cycles)
        else:
            e.rs_norm(self.grads.ptrs, self.signals.ptrs, self.rank, shard_lo, shard_n, grad_shard, self.epoch,
                      self.status, self.wait_cycles)
        ev[1].record()
        args = (self.signals.ptrs, self.rank, shard_lo, shard_n, master, grad_shard, m, v, lr, betas[0], betas[1], eps,
                wd, step, max_norm if max_norm else 0.0, self.epoch, self.status, self.norm, self.wait_cycles)
        if self.nvls:
            e.adamw_ag_mc(self.weights.mc, *args)
        else:
            e.adamw_ag(self.weights.ptrs, *args)
        ev[2].record()
        vals = torch.cat([self.norm, self.status.float()]).cpu()   # one device->host read per step
        # device time of the two kernels (the read above waited for both)
        self.last_timing = {"opt_rs_s": ev[0].elapsed_time(ev[1]) / 1e3,
                            "opt_bcast_s": ev[1].elapsed_time(ev[2]) / 1e3}
        norm, status = float(vals[0]), int(vals[1])
        if status:
            raise CommTimeout(f"fused optimizer step: a cross-rank wait expired (code {status}); "
                              "a peer rank is dead or stalled")
        return norm, not (norm == norm and norm != float("inf"))

    def check(self) -> None:
        s = int(self.status.item())
        if s:
            raise CommTimeout(f"cross-rank wait expired (code {s})")

    def close(self) -> None:
        for b in (self.weights, self.grads, self.signals):
            b.close()


class NVLinkAllReduce:
    """All-reduce for replicated data parallel (the draft model of the SDDD
    layout, DDP-style replicas) on this package's NVLink kernel instead of
    NCCL: the bucket is staged in an fp32 symmetric buffer, one kernel sums
    every rank's copy slice by slice over peer memory and writes the result
    into every copy (``nvls``: the NVLS multimem variant, opt-in like the
    optimizer's), and the result is read back.  Sums run in fp32 whatever the
    gradient dtype.  Every cross-rank wait is bounded: a dead or late peer
    raises ``CommTimeout``."""

    def __init__(self, capacity: int, rank: int, world: int, group=None, wait_seconds: float = 10.0,
                 nvls: Optional[bool] = None) -> None:
        self.capacity = (capacity + 3) // 4 * 4
        self.rank, self.world, self.group = rank, world, group
        self.wait_cycles = int(wait_seconds * 2.0e9)
        if nvls is None:
            nvls = os.environ.get("LRL_NVLS", "0") == "1"
        self.nvls = False
        if nvls and nvls_supported():
            self.buf = MulticastBuffer(self.capacity, torch.float32, group)
            self.nvls = self.buf.mc != 0
            if not self.nvls:
                self.buf.close()
        if not self.nvls:
            self.buf = SymmetricBuffer(self.capacity, torch.float32, rank, world, group)
        self.signals = SymmetricBuffer(int(ext().symm_signal_words()), torch.int32, rank, world, group)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.buf.tensor.device)
        self.epoch = 0
        dist.barrier(group=group)

    def all_reduce_(self, flat: torch.Tensor, scale: float = 1.0) -> torch.Tensor:
        """In place: ``flat`` (1-D, any float dtype) <- scale * sum over ranks.
        Buckets larger than the buffer go through it in pieces."""
        n = flat.numel()
        for a in range(0, n, self.capacity):
            b = min(n, a + self.capacity)
            m = b - a
            m4 = (m + 3) // 4 * 4
            stage = self.buf.tensor[:m4]
            stage[:m].copy_(flat[a:b])
            if m4 != m:
                stage[m:].zero_()
            self.epoch += 1
            if self.nvls:
                ext().nvlink_allreduce_mc(self.buf.mc, self.signals.ptrs, self.rank, m4, scale, self.epoch,
                                          self.status, self.wait_cycles)
            else:
                ext().nvlink_allreduce(self.buf.ptrs, self.signals.ptrs, self.rank, m4, scale, self.epoch,
                                       self.status, self.wait_cycles)
            flat[a:b].copy_(stage[:m])
        return flat

    def check(self) -> None:
        """Raise ``CommTimeout`` if a cross-rank wait of an earlier call expired
        (one device->host read)."""
        s = int(self.status.item())
        if s:
            raise CommTimeout(f"NVLink all-reduce: a cross-rank wait expired (code {s}); a peer rank is dead or stalled")

    def close(self) -> None:
        torch.cuda.synchronize()
        self.buf.close()
        self.signals.close()


# ---------------------------------------------------------------------------
# correctness checks of the data-parallel replicas (used by bench.py at N > 1
# and by the multi-GPU tests)
# ---------------------------------------------------------------------------

def _bits_checksum(t: torch.Tensor, chunk: int = 1 << 26) -> tuple[int, int]:
    """Order-sensitive checksum of a tensor's bit pattern: (sum of the 16-bit
    words, sum of word x (index mod 65521)); identical bytes give identical
    pairs on every rank."""
    w = t.reshape(-1).view(torch.int16)
    s0 = s1 = 0
    for a in range(0, w.numel(), chunk):
        x = w[a: a + chunk].to(torch.int64) & 0xFFFF
        idx = (torch.arange(a, a + x.numel(), device=x.device, dtype=torch.int64) % 65521)
        s0 += int(x.sum())
        s1 += int((x * idx).sum())
    return s0, s1


def replica_agreement(model_flat: torch.Tensor, master: torch.Tensor, lo: int, group=None) -> dict:
    """Do all ranks hold bit-identical resident bf16 weights, and does every
    rank's bf16 slice equal its fp32 master shard rounded to bf16?"""
    world = dist.get_world_size(group)
    cs = _bits_checksum(model_flat)
    own = model_flat[lo: lo + master.numel()]
    mism = int((master.to(own.dtype).view(torch.int16) != own.view(torch.int16)).sum())
    mine = torch.tensor([cs[0], cs[1], mism], dtype=torch.int64, device=model_flat.device)
    every = [torch.zeros_like(mine) for _ in range(world)]
    dist.all_gather(every, mine, group=group)
    rows = [tuple(int(v) for v in e.tolist()) for e in every]
    same = all(r[:2] == rows[0][:2] for r in rows)
    return {"ranks_agree": bool(same and all(r[2] == 0 for r in rows)), "weights_identical": bool(same),
            "master_mismatches": sum(r[2] for r in rows)}


def fused_vs_nccl_max_err(numel: int, rank: int, world: int, steps: int = 1, group=None, seed: int = 0,
                          nvls: Optional[bool] = None) -> dict:
    """One (or more) fused NVLink optimizer steps (rs_norm + adamw_ag) against
    NCCL reduce_scatter_tensor + the AdamW kernel + all_gather_into_tensor on
    the same gradients; returns the largest differences of the resulting bf16
    weights and fp32 master shards.  Allocates ~``numel`` x 14 bytes per rank."""
    from lumenrl_b200.engine.training.optimizer import ShardedFlatAdamW
    n = max(numel // (world * 128), 1) * world * 128
    dev = torch.device("cuda", torch.cuda.current_device())
    g0 = torch.Generator(device=dev).manual_seed(seed)
    w0 = torch.randn(n, device=dev, generator=g0).to(torch.bfloat16)
    comm = NVLinkOptimizerComm(n, rank, world, group=group, nvls=nvls)
    try:
        comm.weights.tensor.copy_(w0)
        kw = dict(lr=1e-3, betas=(0.9, 0.95), weight_decay=0.1, max_grad_norm=1.0)
        fused = ShardedFlatAdamW(comm.weights.tensor, world, rank, comm=comm, **kw)
        plain_w = w0.clone()
        plain = ShardedFlatAdamW(plain_w, world, rank, **kw)
        norm_err = 0.0
        for s in range(steps):
            g = torch.randn(n, device=dev, generator=torch.Generator(device=dev).manual_seed(seed + 1000 * s + rank))
            fused.grad.copy_(g)
            plain.grad.copy_(g)
            a, b = fused.step(), plain.step()
            norm_err = max(norm_err, abs(a["grad_norm"] - b["grad_norm"]) / max(1.0, b["grad_norm"]))
        torch.cuda.synchronize()
        out = torch.tensor([(comm.weights.tensor.float() - plain_w.float()).abs().max().item(),
                            (fused.master - plain.master).abs().max().item(), norm_err], device=dev)
        dist.all_reduce(out, op=dist.ReduceOp.MAX, group=group)
        return {"weights_max_err": float(out[0]), "master_max_err": float(out[1]), "grad_norm_rel_err": float(out[2]),
                "numel": n, "nvls": comm.nvls}
    finally:
        torch.cuda.synchronize()
        dist.barrier(group=group)
        comm.close()
