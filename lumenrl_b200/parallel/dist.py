"""Process-group plumbing: one process per GPU, NCCL for CUDA, gloo for CPU.

``init_distributed`` reads the torchrun environment (RANK, WORLD_SIZE,
LOCAL_RANK, MASTER_ADDR/PORT), uses a short timeout so a dead peer ends a
collective with an error instead of a hang, and pins the device.
``ParallelState`` records the data/tensor/expert/pipeline/context groups.
"""

from __future__ import annotations

import datetime
import os
from dataclasses import dataclass, field
from typing import Optional

import torch
import torch.distributed as dist


@dataclass
class ParallelState:
    world_size: int = 1
    rank: int = 0
    local_rank: int = 0
    device: torch.device = field(default_factory=lambda: torch.device("cpu"))
    dp_group: Optional[object] = None
    tp_size: int = 1
    ep_size: int = 1
    pp_size: int = 1
    cp_size: int = 1
    # context parallelism: ranks of one CP group hold the same rows and split
    # every sequence into zigzag chunks (parallel/context_parallel.py)
    cp_group: Optional[object] = None
    cp_rank: int = 0

    @property
    def dp_size(self) -> int:
        return self.world_size // (self.tp_size * self.pp_size * self.cp_size)

    @property
    def is_distributed(self) -> bool:
        return self.world_size > 1


_STATE = ParallelState()


def get_state() -> ParallelState:
    return _STATE


def init_distributed(backend: Optional[str] = None, timeout_s: float = 600.0, device: Optional[str] = None) -> ParallelState:
    global _STATE
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    use_cuda = (device or ("cuda" if torch.cuda.is_available() else "cpu")).startswith("cuda")
    if use_cuda:
        torch.cuda.set_device(local)
        dev = torch.device("cuda", local)
    else:
        dev = torch.device("cpu")
    if world > 1 and not dist.is_initialized():
        be = backend or ("nccl" if use_cuda else "gloo")
        kw = {}
        if use_cuda and be == "nccl":
            kw["device_id"] = dev
        dist.init_process_group(backend=be, timeout=datetime.timedelta(seconds=timeout_s), **kw)
    _STATE = ParallelState(world_size=world, rank=rank, local_rank=local, device=dev)
    return _STATE


def set_state(st: ParallelState) -> ParallelState:
    """Make ``st`` the process's state: the scalar collectives below then run
    on ``st.dp_group`` (a sub-group, e.g. the trainer ranks of a separated
    trainer / rollout layout)."""
    global _STATE
    _STATE = st
    return st


def sub_state(ranks: list[int], group) -> ParallelState:
    """State of this process inside ``group`` (built over global ``ranks``):
    group-local rank and size, same device."""
    me = dist.get_rank()
    return ParallelState(world_size=len(ranks), rank=ranks.index(me), local_rank=_STATE.local_rank,
                         device=_STATE.device, dp_group=group)


def barrier() -> None:
    if dist.is_initialized():
        dist.barrier(group=_STATE.dp_group)


def all_reduce_max(x: float) -> float:
    if not dist.is_initialized():
        return x
    t = torch.tensor([x], dtype=torch.float64, device=_STATE.device if _STATE.device.type == "cuda" else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=_STATE.dp_group)
    return float(t.item())


def all_reduce_sum(x: float, state: Optional[ParallelState] = None) -> float:
    """Sum of ``x`` over the data-parallel group of ``state`` (default: the
    process-wide state); a single-rank state sums nothing."""
    st = state if state is not None else _STATE
    if not dist.is_initialized() or (state is not None and state.world_size == 1):
        return x
    t = torch.tensor([x], dtype=torch.float64, device=st.device if st.device.type == "cuda" else "cpu")
    dist.all_reduce(t, group=st.dp_group)
    return float(t.item())


def _reduce_many(xs: list, op) -> list:
    if not dist.is_initialized() or not xs:
        return [float(x) for x in xs]
    t = torch.tensor([float(x) for x in xs], dtype=torch.float64,
                     device=_STATE.device if _STATE.device.type == "cuda" else "cpu")
    dist.all_reduce(t, op=op, group=_STATE.dp_group)
    return t.tolist()


def all_reduce_sum_many(xs: list) -> list:
    """Element-wise sum over the data-parallel group of several host scalars
    in ONE collective (and one device->host read)."""
    return _reduce_many(xs, dist.ReduceOp.SUM)


def all_reduce_max_many(xs: list) -> list:
    """Element-wise max over the data-parallel group in one collective."""
    return _reduce_many(xs, dist.ReduceOp.MAX)


def destroy() -> None:
    if dist.is_initialized():
        dist.destroy_process_group()
