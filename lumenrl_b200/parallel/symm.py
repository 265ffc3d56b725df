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

Waits are bounded in the kernels; ``check()`` raises ``CommTimeout`` when a
kernel recorded an expired wait (a dead or stalled rank).
"""

from __future__ import annotations

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


class NVLinkOptimizerComm:
    """Fused reduce-scatter / AdamW / all-gather over NVLink peer memory."""

    def __init__(self, numel: int, rank: int, world: int, weight_dtype=torch.bfloat16, group=None,
                 wait_seconds: float = 10.0) -> None:
        self.rank, self.world, self.group = rank, world, group
        # in-kernel spin bound, in SM clock cycles at boost clock
        self.wait_cycles = int(wait_seconds * 2.0e9)
        self.weights = SymmetricBuffer(numel, weight_dtype, rank, world, group)
        self.grads = SymmetricBuffer(numel, torch.float32, rank, world, group)
        self.signals = SymmetricBuffer(int(ext().symm_signal_words()), torch.int32, rank, world, group)
        dev = self.weights.tensor.device
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        self.norm = torch.zeros(1, dtype=torch.float32, device=dev)
        self.epoch = 0
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
        e.rs_norm(self.grads.ptrs, self.signals.ptrs, self.rank, shard_lo, shard_n, grad_shard, self.epoch,
                  self.status, self.wait_cycles)
        e.adamw_ag(self.weights.ptrs, self.signals.ptrs, self.rank, shard_lo, shard_n, master, grad_shard, m, v, lr,
                   betas[0], betas[1], eps, wd, step, max_norm if max_norm else 0.0, self.epoch, self.status,
                   self.norm, self.wait_cycles)
        vals = torch.cat([self.norm, self.status.float()]).cpu()   # one device->host read per step
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
