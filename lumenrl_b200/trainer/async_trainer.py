"""Fully-async RL: rollout and training overlap with bounded staleness.

Reference: ``lumenrl/trainer/async_trainer.py:58-790`` and
``message_queue.py:28-139``.  A producer (``Rollouter``) generates batches
with the current rollout weights and tags each with the parameter version
that produced it; the trainer consumes ``require_batches`` batches per update
from a bounded ``AsyncMessageQueue`` that drops samples older than the
allowed staleness (``staleness_threshold`` = fraction of stale samples a
batch may contain), and every ``trigger_parameter_sync_step`` updates pushes
new weights to the rollouter (bumping ``param_version``).

On one process the rollouter runs on a background thread with its own CUDA
stream and its own weight copy (separated mode); rollout log-probs are used
as old log-probs when ``use_rollout_log_probs`` (the off-policy ratio then
measures real staleness, corrected by TIS when enabled).
"""

from __future__ import annotations

import logging
import queue
import threading
import time
from dataclasses import dataclass, field
from typing import Optional

import torch

from lumenrl_b200.core.protocol import DataProto
from lumenrl_b200.trainer.rl_trainer import RLTrainer

logger = logging.getLogger(__name__)


@dataclass
class SampleItem:
    data: DataProto
    param_version: int = 0
    created_at: float = field(default_factory=time.time)


class AsyncMessageQueue:
    def __init__(self, maxsize: int = 64, staleness_threshold: float = 0.0) -> None:
        self._q: "queue.Queue[SampleItem]" = queue.Queue(maxsize=maxsize)
        self.staleness_threshold = staleness_threshold
        self._version = 0
        self._lock = threading.Lock()
        self.produced = self.consumed = self.stale_consumed = self.dropped = 0

    @property
    def current_param_version(self) -> int:
        return self._version

    @current_param_version.setter
    def current_param_version(self, v: int) -> None:
        with self._lock:
            self._version = v

    def put(self, item: SampleItem, timeout: Optional[float] = None) -> None:
        self._q.put(item, timeout=timeout)
        with self._lock:
            self.produced += 1

    def get_batch(self, batch_size: int, timeout: float = 300.0) -> list[SampleItem]:
        out: list[SampleItem] = []
        stale = 0
        max_stale = int(batch_size * self.staleness_threshold)
        deadline = time.monotonic() + timeout
        while len(out) < batch_size:
            left = deadline - time.monotonic()
            if left <= 0:
                raise TimeoutError(f"AsyncMessageQueue.get_batch timed out: got {len(out)}/{batch_size} in {timeout}s")
            try:
                item = self._q.get(timeout=min(left, 1.0))
            except queue.Empty:
                continue
            if item.param_version < self._version:
                if stale >= max_stale:
                    with self._lock:
                        self.dropped += 1
                    continue
                stale += 1
            out.append(item)
        with self._lock:
            self.consumed += len(out)
            self.stale_consumed += stale
        return out

    def qsize(self) -> int:
        return self._q.qsize()

    def stats(self) -> dict:
        return {"async/produced": self.produced, "async/consumed": self.consumed,
                "async/stale_consumed": self.stale_consumed, "async/dropped": self.dropped,
                "async/queue_size": self.qsize(), "async/param_version": self._version}


class AsyncRLTrainer(RLTrainer):
    """Trainer + background rollouter on a separate weight copy."""

    def setup(self) -> "AsyncRLTrainer":
        super().setup()
        ac = self.config.async_training
        self.mq = AsyncMessageQueue(ac.queue_maxsize, ac.staleness_threshold)
        from lumenrl_b200.engine.inference.engine import RolloutEngine
        from lumenrl_b200.models.qwen3 import Qwen3Model
        st = self.state
        dtype = self.actor.model.flat.dtype
        self.rollout_model = Qwen3Model(self.model_args, device=st.device, dtype=dtype, requires_grad=False)
        self.rollout_model.flat.copy_(self.actor.model.flat)
        # the base class built a colocated engine on the actor's buffer: free its
        # KV pool before the separated engine (own weight copy) replaces it
        self.rollout.sleep(release_memory=True)
        self.rollout = RolloutEngine(self.rollout_model, max_num_seqs=self.prompts_per_rank * self.group,
                                     max_model_len=self.spec.prompt_len + self.spec.max_new_tokens,
                                     use_cuda_graph=False)
        self._stop = threading.Event()
        self._rollout_step = 0
        self._weights_lock = threading.Lock()
        self._stream = torch.cuda.Stream() if st.device.type == "cuda" else None
        self._thread: Optional[threading.Thread] = None
        self._sync_every = max(1, ac.trigger_parameter_sync_step)
        self._updates = 0
        return self

    def _rollout_loop(self) -> None:
        while not self._stop.is_set():
            with self._weights_lock:
                version = self.mq.current_param_version
                if self._stream is not None:
                    with torch.cuda.stream(self._stream):
                        batch = self._rollout(self._rollout_step)
                    self._stream.synchronize()
                else:
                    batch = self._rollout(self._rollout_step)
            self._rollout_step += 1
            try:
                self.mq.put(SampleItem(batch, version), timeout=1.0)
            except queue.Full:
                if self._stop.is_set():
                    return

    def start_rollouter(self) -> None:
        if self._thread is None:
            self._thread = threading.Thread(target=self._rollout_loop, daemon=True)
            self._thread.start()

    def stop_rollouter(self) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=60)
            self._thread = None

    def step(self) -> dict:
        self.start_rollouter()
        ac = self.config.async_training
        items = self.mq.get_batch(max(1, ac.require_batches))
        batch = DataProto.concat([it.data for it in items])
        batch.meta = dict(items[0].data.meta)
        batch.meta["uid"] = [u for it in items for u in it.data.meta["uid"]]
        m = self._train_on(batch, use_rollout_logprobs=ac.use_rollout_log_probs)
        self._updates += 1
        if self._updates % self._sync_every == 0:
            t0 = time.perf_counter()
            with self._weights_lock:
                self.rollout_model.flat.copy_(self.actor.model.flat)
                self.mq.current_param_version = self.mq.current_param_version + 1
            m["weight_sync/ms"] = (time.perf_counter() - t0) * 1e3
        m.update(self.mq.stats())
        m["staleness/mean_version_lag"] = sum(self.mq.current_param_version - it.param_version for it in items) / len(items)
        self.global_step += 1
        self.history.append(m)
        return m

    def _train_on(self, batch: DataProto, use_rollout_logprobs: bool) -> dict:
        st = self.state
        rewards = self.reward_fn(batch["responses"], None, lengths=batch["response_lengths"], **self.spec.reward_kwargs)
        batch["rewards"] = rewards.to(st.device).float()
        if use_rollout_logprobs:
            batch["old_log_probs"] = batch["rollout_log_probs"]
        else:
            batch["old_log_probs"], _ = self.actor.compute_log_probs(batch, self.temperature)
        self.algorithm.compute_advantages(batch)
        pol = self.config.algorithm.dapo if self.algorithm_name == "dapo" else self.algo_cfg
        m = self.actor.update_policy(batch, pol, self.algorithm_name, rows_per_micro=self.spec.rows_per_micro,
                                     temperature=self.temperature)
        m["reward/mean"] = float(batch["rewards"].mean())
        m["step"] = self.global_step + 1
        return m

    def cleanup(self) -> None:
        self.stop_rollouter()
        super().cleanup()
