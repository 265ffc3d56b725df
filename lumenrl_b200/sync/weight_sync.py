"""Trainer -> rollout weight synchronisation.

Backends (``weight_sync.backend``; reference ``rl_trainer.py:729-915``,
``engine/training/weight_sync.py``, ``trainer/weight_sync.py``):

* ``inplace`` (colocated, same GPU): the rollout engine reads the trainer's
  resident bf16 buffer; sync is a version bump.  On several GPUs the fused
  optimizer kernel already stored every rank's new shard into every rank's
  buffer (``parallel.symm``), so nothing else moves.
* ``broadcast`` (separated trainer/rollout GPU groups on one node): the flat
  bf16 buffer is broadcast in ``bucket_size_mb`` chunks from a trainer rank
  to rollout ranks over the process group (NCCL over NVLink), optionally with
  blockwise FP8 requantisation on the receiving side.
* ``p2p`` (separated, one node): the trainer rank stores its flat bf16
  buffer straight into the rollout rank's IPC-mapped weight buffer with the
  ``p2p_push`` copy kernel (plain NVLink stores in bucket-sized launches, a
  ready flag per bucket), and the receiver waits on the flags (bounded) and
  re-quantises FP8 rollout weights if it runs them.  The receiver acknowledges
  each version when it asks for the next, and the sender waits for that
  acknowledgement before pushing, so weights in use are never overwritten.
* ``shared_folder``: safetensors snapshots ``v<N>/`` with a version file on a
  shared filesystem (the reference's FilesystemWeightSync), for cross-node or
  fully-async rollout.
Every sync reports ``weight_sync/ms`` and ``weight_sync/GBps``.
"""

from __future__ import annotations

import os
import shutil
import time
from pathlib import Path
from typing import Optional

import torch
import torch.distributed as dist


class InPlaceWeightSync:
    def __init__(self, engine) -> None:
        self.engine = engine
        self.version = 0

    def sync(self, flat: Optional[torch.Tensor] = None) -> dict:
        t0 = time.perf_counter()
        self.version += 1
        self.engine.update_weights(flat, self.version)
        nbytes = 0 if flat is None or flat.data_ptr() == self.engine.model.flat.data_ptr() else flat.numel() * 2
        dt = time.perf_counter() - t0
        return {"weight_sync/ms": dt * 1e3, "weight_sync/GBps": nbytes / max(dt, 1e-9) / 1e9,
                "weight_sync/version": self.version}


class BroadcastWeightSync:
    """Chunked broadcast of the flat weights from ``src`` to a group."""

    def __init__(self, flat: torch.Tensor, src: int, group=None, bucket_size_mb: int = 1024,
                 requant_fp8: bool = False) -> None:
        self.flat, self.src, self.group = flat, src, group
        self.bucket = max(1, bucket_size_mb * 1024 * 1024 // flat.element_size())
        self.requant_fp8 = requant_fp8
        self.version = 0

    def sync(self) -> dict:
        t0 = time.perf_counter()
        n = self.flat.numel()
        for a in range(0, n, self.bucket):
            dist.broadcast(self.flat[a: min(n, a + self.bucket)], src=self.src, group=self.group)
        if self.flat.is_cuda:
            torch.cuda.synchronize()
        self.version += 1
        dt = time.perf_counter() - t0
        return {"weight_sync/ms": dt * 1e3, "weight_sync/GBps": n * self.flat.element_size() / max(dt, 1e-9) / 1e9,
                "weight_sync/version": self.version}


class P2PWeightSync:
    """Trainer rank ``src`` -> rollout rank ``dst`` over NVLink peer stores.

    Both ranks construct it (collectively over ``group``); ``dst`` passes its
    rollout engine.  The receiver's flat weights live in a symmetric buffer,
    so the rollout model is re-pointed at it once at construction."""

    def __init__(self, numel: int, src: int, dst: int, group=None, engine=None, bucket_size_mb: int = 1024,
                 wait_seconds: float = 30.0) -> None:
        from lumenrl_b200.ops.ext import ext
        from lumenrl_b200.parallel.symm import SymmetricBuffer
        self.src, self.dst, self.group = src, dst, group
        self.rank = dist.get_rank(group)
        world = dist.get_world_size(group)
        self._e = ext()
        self.buf = SymmetricBuffer(numel, torch.bfloat16, self.rank, world, group)
        # words 0..63 on the receiver: bucket-ready flags; word 64 on the
        # sender: the receiver's "done with version v" acknowledgement
        self.sig = SymmetricBuffer(128, torch.int32, self.rank, world, group)
        self.bucket = max(8, (bucket_size_mb * 1024 * 1024 // 2) // 8 * 8)
        self.numel = numel
        dev = self.buf.tensor.device
        self.counter = torch.zeros(1, dtype=torch.int32, device=dev)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        self.wait_cycles = int(wait_seconds * 2.0e9)
        self.version = 0
        self.engine = engine
        if engine is not None and self.rank == dst:
            self.buf.tensor.copy_(engine.model.flat)
            engine.model.flat = self.buf.tensor   # later syncs land in place
            for name, p in engine.model.named_flat_params():
                p.data = engine.model.layout.view(self.buf.tensor, name)
        dist.barrier(group=group)

    def sync(self, flat: Optional[torch.Tensor] = None) -> dict:
        """``src`` passes its flat bf16 weights; ``dst`` passes nothing."""
        t0 = time.perf_counter()
        self.version += 1
        e = self._e
        if self.rank == self.src:
            assert flat is not None and flat.numel() == self.numel and flat.dtype == torch.bfloat16
            # back-pressure: never overwrite weights the rollout side still uses
            e.p2p_wait(self.sig.ptrs[self.src] + 4 * 64, self.version - 1, self.status, 4, self.wait_cycles)
            nb = (self.numel + self.bucket - 1) // self.bucket
            for i in range(nb):
                a, b = i * self.bucket, min(self.numel, (i + 1) * self.bucket)
                # flag word i % 64 carries the bucket's version
                e.p2p_push(flat[a:b], self.buf.ptrs[self.dst] + 2 * a, self.sig.ptrs[self.dst] + 4 * (i % 64),
                           self.version, self.counter)
            torch.cuda.synchronize()
            if int(self.status.item()):
                from lumenrl_b200.parallel.symm import CommTimeout
                raise CommTimeout("p2p weight sync: the rollout side never released the previous weights")
        elif self.rank == self.dst:
            # release the previous version (the caller is done generating with it)
            e.p2p_signal(self.sig.ptrs[self.src] + 4 * 64, self.version - 1)
            # the sender's pushes run in stream order and each publishes its flag
            # with a system-scope release after its stores, so the last
            # bucket's flag implies every bucket has landed
            nb = (self.numel + self.bucket - 1) // self.bucket
            e.p2p_wait(self.sig.ptrs[self.dst] + 4 * ((nb - 1) % 64), self.version, self.status, 3,
                       self.wait_cycles)
            torch.cuda.synchronize()
            if int(self.status.item()):
                from lumenrl_b200.parallel.symm import CommTimeout
                raise CommTimeout("p2p weight sync: the trainer never delivered a bucket")
            if self.engine is not None:
                self.engine.update_weights(version=self.version)
        dt = time.perf_counter() - t0
        return {"weight_sync/ms": dt * 1e3, "weight_sync/GBps": self.numel * 2 / max(dt, 1e-9) / 1e9,
                "weight_sync/version": self.version}

    def close(self) -> None:
        torch.cuda.synchronize()
        self.buf.close()
        self.sig.close()


class FilesystemWeightSync:
    def __init__(self, sync_dir: str, keep_versions: int = 2) -> None:
        self.dir = Path(sync_dir)
        self.dir.mkdir(parents=True, exist_ok=True)
        self.keep = keep_versions
        self.version = 0

    def push(self, state_dict: dict[str, torch.Tensor], version: Optional[int] = None) -> str:
        from safetensors.torch import save_file
        self.version = self.version + 1 if version is None else version
        d = self.dir / f"v{self.version}"
        d.mkdir(parents=True, exist_ok=True)
        save_file({k: v.detach().contiguous().cpu() for k, v in state_dict.items()}, str(d / "model.safetensors"))
        (d / "version.txt").write_text(str(self.version))
        for old in sorted(self.dir.glob("v*"), key=lambda p: int(p.name[1:]) if p.name[1:].isdigit() else -1):
            if old.name[1:].isdigit() and int(old.name[1:]) <= self.version - self.keep:
                shutil.rmtree(old, ignore_errors=True)
        return str(d)

    def latest_path(self) -> Optional[str]:
        vs = [int(p.name[1:]) for p in self.dir.glob("v*") if p.name[1:].isdigit() and (p / "version.txt").exists()]
        return str(self.dir / f"v{max(vs)}") if vs else None

    def pull(self) -> tuple[Optional[dict], int]:
        p = self.latest_path()
        if p is None:
            return None, 0
        from safetensors.torch import load_file
        return load_file(os.path.join(p, "model.safetensors")), int(Path(p, "version.txt").read_text())
