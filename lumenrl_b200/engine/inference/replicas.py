"""Rollout replicas behind HTTP: server, replica manager, load-balancing client.

The in-process ``RolloutEngine`` is the default rollout path.  This module
serves the same engine as independent replicas -- one process per GPU, each
with its own HTTP endpoint -- for rollout fleets that live outside the
trainer's process group (separate jobs, other hosts, a serving tier), the role
the reference fills with Ray actors wrapping vLLM/ATOM servers
(``lumenrl/engine/inference/vllm_ray_server.py:391-713``) and a driver-side
request router (``vllm_http_engine.py:17-100``).

* ``ReplicaServer`` (one per process): an aiohttp application around one
  ``RolloutEngine``.  Token ids in, token ids + rollout log-probs (+ routed
  expert ids of MoE models, for R3) out; msgpack bodies.
  ``POST /generate``, ``/sleep``, ``/wake``, ``/drain``, ``/reload_weights``
  (an HF-named safetensors file or directory, e.g. one written by
  ``FilesystemWeightSync.push``), ``GET /health``.
* ``ReplicaManager``: starts N replica processes (``spawn``), each pinned to
  one device, waits until they answer, and fans the control calls out
  (``sleep_all`` / ``wake_all`` / ``drain_all`` / ``reload_weights_from_path``
  / ``shutdown``).
* ``RolloutClient``: splits a prompt batch into contiguous slices, one per
  replica, posts them concurrently and reassembles the rows in order.  Each
  slice carries its global row offset, so the samples (counter-based streams
  keyed by global row and token index) equal one engine's on the whole batch.
* ``HttpRolloutEngine``: the trainer-facing adapter (``generate_tokens``,
  ``generate`` returning a ``GenerationOutput``, ``sleep``, ``wake``,
  ``update_weights_from_path``, ``shutdown``).
"""

from __future__ import annotations

import asyncio
import logging
import multiprocessing as mp
import os
import threading
from concurrent.futures import ThreadPoolExecutor
from dataclasses import asdict
from typing import Any, Optional

import msgpack
import torch

from lumenrl_b200.engine.inference.engine import GenerationOutput, SamplingParams

logger = logging.getLogger(__name__)

_MSGPACK = "application/msgpack"


def _pack(obj: Any) -> bytes:
    return msgpack.packb(obj, use_bin_type=True)


def _unpack(data: bytes) -> Any:
    return msgpack.unpackb(data, raw=False)


def _tensor_blob(t: torch.Tensor) -> dict:
    t = t.detach().cpu().contiguous()
    return {"dtype": str(t.dtype).replace("torch.", ""), "shape": list(t.shape), "data": t.numpy().tobytes()}


def _blob_tensor(b: dict) -> torch.Tensor:
    import numpy as np
    dt = {"int16": np.int16, "int32": np.int32, "int64": np.int64, "float32": np.float32}[b["dtype"]]
    return torch.from_numpy(np.frombuffer(b["data"], dtype=dt).copy()).view(b["shape"])


# ---------------------------------------------------------------------------------------------- server
class ReplicaServer:
    """One rollout engine behind an HTTP endpoint."""

    def __init__(self, engine, replica_id: int = 0) -> None:
        self.engine = engine
        self.replica_id = replica_id
        self.inflight = 0
        self.sleeping = False
        self._lock = asyncio.Lock()          # one generation at a time on the engine
        self._idle = asyncio.Event()
        self._idle.set()

    def app(self):
        from aiohttp import web
        app = web.Application(client_max_size=1 << 30)
        app.router.add_get("/health", self.health)
        app.router.add_post("/generate", self.generate)
        app.router.add_post("/sleep", self.sleep)
        app.router.add_post("/wake", self.wake)
        app.router.add_post("/drain", self.drain)
        app.router.add_post("/reload_weights", self.reload_weights)
        return app

    @staticmethod
    def _reply(obj: dict):
        from aiohttp import web
        return web.Response(body=_pack(obj), content_type=_MSGPACK)

    async def health(self, request):
        return self._reply({"ok": True, "replica": self.replica_id, "weight_version": self.engine.weight_version,
                            "sleeping": self.sleeping, "inflight": self.inflight})

    async def generate(self, request):
        req = _unpack(await request.read())
        sp = SamplingParams(**req.get("sampling", {}))
        prompts = [list(map(int, p)) for p in req["prompts"]]
        self.inflight += 1
        self._idle.clear()
        try:
            async with self._lock:
                out = await asyncio.get_running_loop().run_in_executor(None, self.engine.generate, prompts, sp)
        finally:
            self.inflight -= 1
            if self.inflight == 0:
                self._idle.set()
        lens = out.response_lengths.cpu().tolist()
        resp = out.responses.cpu()
        lps = out.logprobs.cpu()
        rows = []
        for i, L in enumerate(lens):
            row = {"prompt_index": int(out.prompt_index[i]), "tokens": resp[i, :L].tolist(),
                   "logprobs": lps[i, :L].tolist()}
            if out.routed_experts:
                row["routed_experts"] = _tensor_blob(out.routed_experts[i])
            rows.append(row)
        return self._reply({"rows": rows, "weight_version": self.engine.weight_version,
                            "stats": {k: float(v) for k, v in out.stats.items() if isinstance(v, (int, float))}})

    async def sleep(self, request):
        req = _unpack(await request.read()) if request.can_read_body else {}
        async with self._lock:
            self.engine.sleep(release_memory=bool(req.get("release_memory", False)))
            self.sleeping = True
        return self._reply({"ok": True})

    async def wake(self, request):
        async with self._lock:
            self.engine.wake()
            self.sleeping = False
        return self._reply({"ok": True})

    async def drain(self, request):
        await self._idle.wait()
        return self._reply({"ok": True})

    async def reload_weights(self, request):
        req = _unpack(await request.read())
        path = req["path"]
        from safetensors.torch import load_file
        files = [path] if os.path.isfile(path) else sorted(
            os.path.join(path, f) for f in os.listdir(path) if f.endswith(".safetensors"))
        if not files:
            return self._reply({"ok": False, "error": f"no safetensors under {path}"})
        sd = {}
        for f in files:
            sd.update(load_file(f))
        async with self._lock:
            self.engine.model.load_hf_state_dict(sd, strict=True)
            self.engine.update_weights(version=req.get("version"))
        return self._reply({"ok": True, "weight_version": self.engine.weight_version})


def _serve(spec: dict, replica_id: int, device: str, ready) -> None:
    """Replica process body: build the model and engine, serve until killed."""
    from aiohttp import web

    from lumenrl_b200.engine.inference.engine import RolloutEngine
    from lumenrl_b200.models.config import ModelArgs
    from lumenrl_b200.models.qwen3 import Qwen3Model
    dev = torch.device(device)
    if dev.type == "cuda":
        torch.cuda.set_device(dev)
    args = ModelArgs(**spec["model_args"])
    dtype = torch.bfloat16 if dev.type == "cuda" else torch.float32
    model = Qwen3Model(args, device=dev, dtype=dtype, requires_grad=False)
    model.init_weights(spec.get("seed", 0))
    engine = RolloutEngine(model, **spec.get("engine_kwargs", {}))
    server = ReplicaServer(engine, replica_id)

    async def main():
        runner = web.AppRunner(server.app())
        await runner.setup()
        site = web.TCPSite(runner, spec.get("host", "127.0.0.1"), 0)
        await site.start()
        port = site._server.sockets[0].getsockname()[1]
        ready.put((replica_id, port))
        while True:
            await asyncio.sleep(3600)

    asyncio.run(main())


# ---------------------------------------------------------------------------------------------- client
class RolloutClient:
    """Contiguous even split of a prompt batch over replicas, posted
    concurrently, rows reassembled in prompt order."""

    def __init__(self, urls: list[str], timeout_s: float = 600.0) -> None:
        if not urls:
            raise ValueError("RolloutClient needs at least one replica URL")
        self.urls = list(urls)
        self.timeout_s = timeout_s
        self._pool = ThreadPoolExecutor(max_workers=max(1, len(urls)))

    def _post(self, url: str, path: str, body: Optional[dict] = None) -> dict:
        import requests
        r = requests.post(url + path, data=_pack(body or {}), headers={"Content-Type": _MSGPACK},
                          timeout=self.timeout_s)
        r.raise_for_status()
        return _unpack(r.content)

    def _get(self, url: str, path: str) -> dict:
        import requests
        r = requests.get(url + path, timeout=self.timeout_s)
        r.raise_for_status()
        return _unpack(r.content)

    def split(self, n_prompts: int) -> list[tuple[int, int]]:
        """[start, end) prompt ranges, one per replica (empty ranges dropped)."""
        k = len(self.urls)
        base, extra = divmod(n_prompts, k)
        out, a = [], 0
        for i in range(k):
            b = a + base + (1 if i < extra else 0)
            out.append((a, b))
            a = b
        return out

    def generate(self, prompts: list[list[int]], sampling: SamplingParams) -> list[dict]:
        n = max(1, sampling.n)
        futs = []
        for url, (a, b) in zip(self.urls, self.split(len(prompts))):
            if b <= a:
                continue
            sp = asdict(sampling)
            sp["row_offset"] = sampling.row_offset + a * n
            futs.append((a, self._pool.submit(self._post, url, "/generate",
                                              {"prompts": prompts[a:b], "sampling": sp})))
        rows: list[dict] = []
        for a, f in futs:
            for r in f.result()["rows"]:
                r["prompt_index"] += a
                rows.append(r)
        rows.sort(key=lambda r: r["prompt_index"])   # stable: samples of a prompt keep their order
        return rows

    def broadcast(self, path: str, body: Optional[dict] = None) -> list[dict]:
        futs = [self._pool.submit(self._post, u, path, body) for u in self.urls]
        return [f.result() for f in futs]

    def health(self) -> list[dict]:
        return [self._get(u, "/health") for u in self.urls]

    def close(self) -> None:
        self._pool.shutdown(wait=False)


# ---------------------------------------------------------------------------------------------- manager
class ReplicaManager:
    """Starts and controls ``num_replicas`` rollout replica processes, one
    per device in ``devices`` (CUDA indices, or ``"cpu"`` entries)."""

    def __init__(self, model_args, devices: list, seed: int = 0, engine_kwargs: Optional[dict] = None,
                 host: str = "127.0.0.1", start_timeout_s: float = 600.0) -> None:
        from dataclasses import asdict as _asdict
        self.spec = {"model_args": _asdict(model_args), "seed": seed, "engine_kwargs": dict(engine_kwargs or {}),
                     "host": host}
        self.devices = [d if isinstance(d, str) else f"cuda:{int(d)}" for d in devices]
        self.host = host
        self.start_timeout_s = start_timeout_s
        self.procs: list = []
        self.urls: list[str] = []
        self.client: Optional[RolloutClient] = None

    @property
    def num_replicas(self) -> int:
        return len(self.devices)

    def create(self) -> "ReplicaManager":
        ctx = mp.get_context("spawn")
        ready = ctx.Queue()
        for i, dev in enumerate(self.devices):
            p = ctx.Process(target=_serve, args=(self.spec, i, dev, ready), daemon=True)
            p.start()
            self.procs.append(p)
        ports = {}
        try:
            for _ in self.devices:
                rid, port = ready.get(timeout=self.start_timeout_s)
                ports[rid] = port
        except Exception:
            self.shutdown()
            raise RuntimeError("rollout replicas did not come up") from None
        self.urls = [f"http://{self.host}:{ports[i]}" for i in range(len(self.devices))]
        self.client = RolloutClient(self.urls)
        return self

    def sleep_all(self, release_memory: bool = False) -> None:
        self.client.broadcast("/sleep", {"release_memory": release_memory})

    def wake_all(self) -> None:
        self.client.broadcast("/wake")

    def drain_all(self) -> None:
        self.client.broadcast("/drain")

    def reload_weights_from_path(self, path: str, version: Optional[int] = None) -> list[int]:
        outs = self.client.broadcast("/reload_weights", {"path": path, "version": version})
        bad = [o for o in outs if not o.get("ok")]
        if bad:
            raise RuntimeError(f"weight reload failed: {bad[0].get('error')}")
        return [int(o["weight_version"]) for o in outs]

    def shutdown(self) -> None:
        if self.client is not None:
            self.client.close()
        for p in self.procs:
            if p.is_alive():
                p.terminate()
        for p in self.procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
        self.procs = []


# ---------------------------------------------------------------------------------------------- adapter
class HttpRolloutEngine:
    """Trainer-facing rollout engine over HTTP replicas."""

    def __init__(self, manager: ReplicaManager, enable_sleep: bool = True) -> None:
        self.manager = manager
        self.client = manager.client
        self.enable_sleep = enable_sleep
        self._lock = threading.Lock()

    def generate_tokens(self, prompts: list[list[int]], sampling: SamplingParams) -> list[dict]:
        return self.client.generate(prompts, sampling)

    def generate(self, prompts, sampling: SamplingParams) -> GenerationOutput:
        """Same result type as ``RolloutEngine.generate`` (host tensors)."""
        if isinstance(prompts, torch.Tensor):
            prompts = prompts.cpu().tolist()
        rows = self.generate_tokens(prompts, sampling)
        width = max([len(r["tokens"]) for r in rows] + [1])
        N = len(rows)
        resp = torch.zeros(N, width, dtype=torch.long)
        lps = torch.zeros(N, width, dtype=torch.float32)
        lens = torch.zeros(N, dtype=torch.long)
        routed = []
        for i, r in enumerate(rows):
            L = len(r["tokens"])
            resp[i, :L] = torch.tensor(r["tokens"], dtype=torch.long)
            lps[i, :L] = torch.tensor(r["logprobs"], dtype=torch.float32)
            lens[i] = L
            if "routed_experts" in r:
                routed.append(_blob_tensor(r["routed_experts"]))
        return GenerationOutput(prompts=[list(p) for p in prompts], responses=resp, response_lengths=lens,
                                logprobs=lps, prompt_index=torch.tensor([r["prompt_index"] for r in rows]),
                                routed_experts=routed)

    def sleep(self, release_memory: bool = False) -> None:
        if self.enable_sleep:
            self.manager.drain_all()
            self.manager.sleep_all(release_memory)

    def wake(self) -> None:
        if self.enable_sleep:
            self.manager.wake_all()

    def update_weights_from_path(self, path: str, version: Optional[int] = None) -> list[int]:
        return self.manager.reload_weights_from_path(path, version)

    def shutdown(self) -> None:
        self.manager.shutdown()
