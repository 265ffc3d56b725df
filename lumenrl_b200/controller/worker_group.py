"""Single-controller worker groups over OS processes (one process per GPU).

The reference drives its roles as Ray actors (``lumenrl/controller/
ray_worker_group.py:36-397``, ``ray_cluster.py:16-164``).  Ray is not part of
this framework; the same controller API runs on ``torch.multiprocessing``:

* ``ResourcePool``: named GPU pools laid out per node (``process_on_nodes``),
  with ``split``/``merge`` and topology tags (separated train/rollout pools).
* ``WorkerGroup``: spawns one process per GPU, constructs the worker class in
  it with RANK/WORLD_SIZE/LOCAL_RANK/MASTER_* set (so the worker can join an
  NCCL group), then serves method calls over a pipe.  Sync and async fan-out,
  ``dispatch_and_call`` (dispatch modes, DP-rank mapping, collect mask),
  liveness, per-call timeouts, and prefixed ``spawn``/``fuse`` views over one
  set of processes (colocated roles).
* Worker-side exceptions come back with their traceback and are re-raised in
  the controller; a worker that dies surfaces as ``WorkerDied``.
"""

from __future__ import annotations

import os
import socket
import time
import traceback
from dataclasses import dataclass, field
from typing import Any, Optional

import torch.multiprocessing as mp

from lumenrl_b200.controller.dispatch import collect_proto, dispatch_proto, dispatch_with_dp_ranks
from lumenrl_b200.core.protocol import DataProto


class WorkerDied(RuntimeError):
    pass


class WorkerCallTimeout(TimeoutError):
    pass


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@dataclass
class ResourcePool:
    name: str
    process_on_nodes: list[int] = field(default_factory=lambda: [1])
    gpu_ids: Optional[list[int]] = None
    topology_tags: dict = field(default_factory=dict)

    def __post_init__(self) -> None:
        if self.gpu_ids is None:
            self.gpu_ids = list(range(sum(self.process_on_nodes)))

    @property
    def world_size(self) -> int:
        return len(self.gpu_ids)

    def split(self, sizes: list[int], names: Optional[list[str]] = None) -> list["ResourcePool"]:
        if sum(sizes) != self.world_size:
            raise ValueError(f"split sizes {sizes} do not add up to {self.world_size}")
        out, lo = [], 0
        for i, s in enumerate(sizes):
            nm = names[i] if names else f"{self.name}_{i}"
            out.append(ResourcePool(nm, [s], self.gpu_ids[lo: lo + s], dict(self.topology_tags)))
            lo += s
        return out

    @staticmethod
    def merge(pools: list["ResourcePool"], name: str = "merged") -> "ResourcePool":
        ids = [g for p in pools for g in p.gpu_ids]
        return ResourcePool(name, [len(ids)], ids)


def _serve(conn, worker_cls, args, kwargs, env: dict) -> None:
    os.environ.update({k: str(v) for k, v in env.items()})
    try:
        worker = worker_cls(*args, **kwargs)
        conn.send(("ok", None))
    except Exception:
        conn.send(("err", traceback.format_exc()))
        return
    while True:
        try:
            msg = conn.recv()
        except EOFError:
            return
        if msg is None:
            return
        method, a, k = msg
        try:
            res = getattr(worker, method)(*a, **k)
            if isinstance(res, DataProto):
                res = res.cpu()
            conn.send(("ok", res))
        except Exception:
            conn.send(("err", traceback.format_exc()))


class _Future:
    def __init__(self, group: "WorkerGroup", idx: int) -> None:
        self.group, self.idx = group, idx

    def get(self, timeout: Optional[float] = None) -> Any:
        return self.group._recv(self.idx, timeout)


class WorkerGroup:
    def __init__(self, worker_cls, pool: ResourcePool, *args, name_prefix: str = "", master_port: Optional[int] = None,
                 extra_env: Optional[dict] = None, start: bool = True, **kwargs) -> None:
        self.worker_cls = worker_cls
        self.pool = pool
        self.args, self.kwargs = args, kwargs
        self.prefix = name_prefix
        self.master_port = master_port or free_port()
        self.extra_env = extra_env or {}
        self._procs: list = []
        self._conns: list = []
        self._shared_from: Optional[WorkerGroup] = None
        if start:
            self.start()

    # ---- lifecycle ----------------------------------------------------------------
    @property
    def world_size(self) -> int:
        return self.pool.world_size

    def start(self) -> None:
        ctx = mp.get_context("spawn")
        n = self.world_size
        for r in range(n):
            parent, child = ctx.Pipe()
            env = {"RANK": r, "WORLD_SIZE": n, "LOCAL_RANK": r, "MASTER_ADDR": "127.0.0.1",
                   "MASTER_PORT": self.master_port, "LUMENRL_WORKER_GPU": self.pool.gpu_ids[r], **self.extra_env}
            p = ctx.Process(target=_serve, args=(child, self.worker_cls, self.args, self.kwargs, env), daemon=True)
            p.start()
            self._procs.append(p)
            self._conns.append(parent)
        for r in range(n):
            self._recv(r, timeout=600)

    def shutdown(self) -> None:
        if self._shared_from is not None:
            return
        for c in self._conns:
            try:
                c.send(None)
            except Exception:
                pass
        for p in self._procs:
            p.join(timeout=10)
            if p.is_alive():
                p.terminate()
        self._procs, self._conns = [], []

    def is_alive(self) -> list[bool]:
        return [p.is_alive() for p in self._procs]

    # ---- calls --------------------------------------------------------------------
    def _send(self, idx: int, method: str, args, kwargs) -> None:
        if not self._procs[idx].is_alive():
            raise WorkerDied(f"worker {idx} of {self.worker_cls.__name__} is dead")
        self._conns[idx].send((self.prefix + method, args, kwargs))

    def _recv(self, idx: int, timeout: Optional[float] = None) -> Any:
        conn = self._conns[idx]
        deadline = None if timeout is None else time.monotonic() + timeout
        while not conn.poll(0.05):
            if not self._procs[idx].is_alive():
                raise WorkerDied(f"worker {idx} of {self.worker_cls.__name__} died (exit {self._procs[idx].exitcode})")
            if deadline is not None and time.monotonic() > deadline:
                raise WorkerCallTimeout(f"worker {idx} did not answer within {timeout}s")
        status, payload = conn.recv()
        if status == "err":
            raise RuntimeError(f"worker {idx} raised:\n{payload}")
        return payload

    def execute_all_async(self, method: str, *args, **kwargs) -> list[_Future]:
        for i in range(self.world_size):
            self._send(i, method, args, kwargs)
        return [_Future(self, i) for i in range(self.world_size)]

    def execute_all_sync(self, method: str, *args, **kwargs) -> list[Any]:
        # drain every worker's answer before raising so no stale reply is left in a pipe
        futs = self.execute_all_async(method, *args, **kwargs)
        out, first_err = [], None
        for f in futs:
            try:
                out.append(f.get())
            except RuntimeError as e:
                out.append(None)
                first_err = first_err or e
        if first_err is not None:
            raise first_err
        return out

    call_all = execute_all_sync

    def execute_rank_zero(self, method: str, *args, **kwargs) -> Any:
        self._send(0, method, args, kwargs)
        return self._recv(0)

    def call_with_timeout(self, method: str, timeout: float, *args, **kwargs) -> list[Any]:
        futs = self.execute_all_async(method, *args, **kwargs)
        return [f.get(timeout=timeout) for f in futs]

    def dispatch_and_call(self, method: str, data: DataProto, mode=None, *, mesh_mapping=None,
                          dp_rank_mapping: Optional[list[int]] = None, collect_mask: Optional[list[bool]] = None,
                          timeout: Optional[float] = None, **kwargs) -> DataProto:
        n = self.world_size
        if dp_rank_mapping is not None:
            chunks = dispatch_with_dp_ranks(data, n, dp_rank_mapping)
        else:
            chunks = dispatch_proto(data, n, mode, mesh_mapping=mesh_mapping)
        targets = list(range(len(chunks)))
        for i in targets:
            self._send(i, method, (chunks[i],), kwargs)
        results = [self._recv(i, timeout) for i in targets]
        if collect_mask is not None:
            results = [r for r, keep in zip(results, collect_mask) if keep]
        return collect_proto(results, mode)

    # ---- prefixed views ------------------------------------------------------------
    def spawn(self, prefixes: list[str]) -> dict[str, "WorkerGroup"]:
        """Views over the SAME processes whose method names get a role prefix
        (``actor_``, ``ref_`` ...) for colocated worker classes."""
        views = {}
        for pre in prefixes:
            v = object.__new__(WorkerGroup)
            v.__dict__.update(self.__dict__)
            v.prefix = f"{pre}_"
            v._shared_from = self
            views[pre] = v
        return views

    fuse = spawn
