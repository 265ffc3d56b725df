"""Hidden-state ring: a producer GPU pushes fixed-size batches straight into a
consumer GPU's memory over NVLink (teacher -> draft hidden states in
speculative-decoding distillation).

Reference counterparts: the MORI-IO store (peer ``copy_`` into an IPC-mapped
buffer plus ``/dev/shm`` ready files with a 60 s timeout,
``lumenrl/transfer/mori_io_store.py:68-303``) and the Mooncake RDMA/TCP KV
store (``transfer/eagle_mooncake_store.py:255-635``).  Here the hand-off is
stream-ordered and stays on the GPUs:

* the consumer owns ``nslots`` slots of ``slot_bytes`` each in a CUDA-IPC
  symmetric buffer, plus a ready flag per slot; the producer owns a free flag
  per slot (both in a small symmetric signal buffer);
* ``put(tensor)`` (producer): waits (bounded, on the GPU) until the consumer
  freed the slot, then ``p2p_push`` copies the rows into the consumer's slot
  with plain stores over NVLink and publishes the slot's epoch in the
  consumer's ready flag;
* ``get(shape, dtype)`` (consumer): waits (bounded) for the ready flag and
  returns a view of the slot; ``release()`` hands the slot back by writing the
  epoch into the producer's free flag.

An expired wait records a status code and ``check()`` raises
``CommTimeout``, so a dead producer or consumer surfaces on the host.  With
no CUDA (or ``backend="pg"``) the same API runs over ``torch.distributed``
send/recv (gloo on CPU), which is what the CPU tests use.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

from lumenrl_b200.parallel.symm import CommTimeout, SymmetricBuffer

# signal words: [0, nslots) ready flags (consumer side), [64, 64 + nslots) free flags (producer side)
_FREE = 64
_SIG_WORDS = 128


class HiddenStateRing:
    def __init__(self, producer: int, consumer: int, slot_bytes: int, nslots: int = 2, group=None,
                 backend: Optional[str] = None, wait_seconds: float = 10.0) -> None:
        if nslots < 1 or nslots > 64:
            raise ValueError("nslots must be in [1, 64]")
        self.producer, self.consumer, self.group = producer, consumer, group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.slot_bytes = (slot_bytes + 255) // 256 * 256
        self.nslots = nslots
        use_cuda = torch.cuda.is_available() and dist.get_backend(group) == "nccl"
        self.backend = backend or ("p2p" if use_cuda else "pg")
        self.sent = 0        # producer: batches pushed
        self.recvd = 0       # consumer: batches taken
        self.wait_cycles = int(wait_seconds * 2.0e9)
        if self.backend == "p2p":
            from lumenrl_b200.ops.ext import ext
            self._ext = ext()
            # collective over the group: every rank maps every peer's buffers
            self.data = SymmetricBuffer(self.slot_bytes * nslots // 4, torch.int32, self.rank, self.world, group)
            self.sig = SymmetricBuffer(_SIG_WORDS, torch.int32, self.rank, self.world, group)
            dev = self.data.tensor.device
            self.status = torch.zeros(1, dtype=torch.int32, device=dev)
            self.counter = torch.zeros(1, dtype=torch.int32, device=dev)
            dist.barrier(group=group)
        self._held: Optional[int] = None

    # ----------------------------------------------------------------- producer
    def put(self, t: torch.Tensor) -> None:
        if self.rank != self.producer:
            raise RuntimeError("put() on a non-producer rank")
        nbytes = t.numel() * t.element_size()
        if nbytes > self.slot_bytes:
            raise ValueError(f"batch of {nbytes} B exceeds the slot size {self.slot_bytes} B")
        i = self.sent
        slot, lap = i % self.nslots, i // self.nslots
        if self.backend == "pg":
            dist.send(t.contiguous(), self._grank(self.consumer), group=self.group)
        else:
            e = self._ext
            if lap > 0:   # wait until the consumer released this slot's previous batch
                e.p2p_wait(self.sig.ptrs[self.rank] + 4 * (_FREE + slot), lap, self.status, 1, self.wait_cycles)
            dst = self.data.ptrs[self.consumer] + slot * self.slot_bytes
            flag = self.sig.ptrs[self.consumer] + 4 * slot
            e.p2p_push(t.contiguous().view(-1), dst, flag, lap + 1, self.counter)
        self.sent += 1

    # ----------------------------------------------------------------- consumer
    def get(self, shape, dtype: torch.dtype, device=None) -> torch.Tensor:
        """Next batch as a ``shape``/``dtype`` tensor.  On the NVLink path this
        is a view of the slot, valid until ``release()``."""
        if self.rank != self.consumer:
            raise RuntimeError("get() on a non-consumer rank")
        if self._held is not None:
            self.release()
        i = self.recvd
        slot, lap = i % self.nslots, i // self.nslots
        numel = 1
        for s in shape:
            numel *= int(s)
        if self.backend == "pg":
            out = torch.empty(*shape, dtype=dtype, device=device or "cpu")
            dist.recv(out, self._grank(self.producer), group=self.group)
            self.recvd += 1
            return out
        e = self._ext
        e.p2p_wait(self.sig.ptrs[self.rank] + 4 * slot, lap + 1, self.status, 2, self.wait_cycles)
        esz = torch.empty(0, dtype=dtype).element_size()
        if numel * esz > self.slot_bytes:
            raise ValueError("requested shape exceeds the slot size")
        words = self.data.tensor.view(torch.uint8)[slot * self.slot_bytes: slot * self.slot_bytes + numel * esz]
        self._held = i
        self.recvd += 1
        return words.view(dtype).view(*shape)

    def release(self) -> None:
        """Hand the slot of the last ``get()`` back to the producer (stream-
        ordered after everything queued that reads it)."""
        if self._held is None or self.backend == "pg":
            self._held = None
            return
        i = self._held
        slot, lap = i % self.nslots, i // self.nslots
        self._ext.p2p_signal(self.sig.ptrs[self.producer] + 4 * (_FREE + slot), lap + 1)
        self._held = None

    # ----------------------------------------------------------------- common
    def check(self) -> None:
        if self.backend == "p2p":
            s = int(self.status.item())
            if s:
                who = "consumer never released a slot" if s == 201 else "producer never pushed"
                raise CommTimeout(f"hidden-state ring wait expired (code {s}): {who}")

    def close(self) -> None:
        if self.backend == "p2p":
            torch.cuda.synchronize()
            self.data.close()
            self.sig.close()

    def _grank(self, r: int) -> int:
        return dist.get_global_rank(self.group, r) if self.group is not None else r
