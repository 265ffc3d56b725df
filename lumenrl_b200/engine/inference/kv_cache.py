"""Paged KV cache and its block allocator.

Layout per layer: ``k[layer]`` and ``v[layer]`` are ``[num_blocks, block_size,
num_kv_heads, head_dim]`` (bf16, or fp8 E4M3 with one scale per layer for
the FP8 KV cache).  A sequence owns a block table (list of block ids); blocks
are reference counted so a GRPO group's G samples share their prompt's full
blocks (prefix sharing) and only the partial tail block is copied per sample.

``sleep()`` frees the pool (colocated training reuses the memory) and
``wake()`` re-allocates it, mirroring the rollout engines' sleep/wake in the
reference (``lumenrl/engine/inference/vllm_engine.py:230-548``).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass
class KVSpec:
    num_layers: int
    num_kv_heads: int
    head_dim: int
    block_size: int = 64
    dtype: torch.dtype = torch.bfloat16

    def bytes_per_block(self) -> int:
        elt = torch.empty(0, dtype=self.dtype).element_size()
        return 2 * self.num_layers * self.block_size * self.num_kv_heads * self.head_dim * elt


class BlockAllocator:
    """Free list + reference counts over ``num_blocks`` ids."""

    def __init__(self, num_blocks: int, reserved: int = 1) -> None:
        # block 0 is reserved: captured CUDA graphs write their warm-up K/V
        # there, so it must never hold a live sequence
        self.num_blocks = num_blocks
        self.free = list(range(num_blocks - 1, reserved - 1, -1))
        self.refs = [0] * num_blocks

    def alloc(self, n: int) -> list[int]:
        if n > len(self.free):
            raise MemoryError(f"KV cache exhausted: need {n} blocks, {len(self.free)} free")
        out = [self.free.pop() for _ in range(n)]
        for b in out:
            self.refs[b] = 1
        return out

    def share(self, blocks: list[int]) -> list[int]:
        for b in blocks:
            self.refs[b] += 1
        return list(blocks)

    def release(self, blocks: list[int]) -> None:
        for b in blocks:
            self.refs[b] -= 1
            if self.refs[b] == 0:
                self.free.append(b)

    @property
    def num_free(self) -> int:
        return len(self.free)


class PagedKVCache:
    def __init__(self, spec: KVSpec, num_blocks: int, device) -> None:
        self.spec = spec
        self.num_blocks = num_blocks
        self.device = torch.device(device)
        self.k: list[torch.Tensor] = []
        self.v: list[torch.Tensor] = []
        self.k_scale = [1.0] * spec.num_layers
        self.v_scale = [1.0] * spec.num_layers
        self.allocator = BlockAllocator(num_blocks)
        self.awake = False
        self.wake()

    @staticmethod
    def blocks_for_budget(spec: KVSpec, budget_bytes: int) -> int:
        return max(1, int(budget_bytes // spec.bytes_per_block()))

    def wake(self) -> None:
        if self.awake:
            return
        s = self.spec
        shape = (self.num_blocks, s.block_size, s.num_kv_heads, s.head_dim)
        # one allocation for all layers so sleep/wake is a single free/malloc
        self._pool = torch.empty((2, s.num_layers) + shape, dtype=s.dtype, device=self.device)
        self.k = [self._pool[0, i] for i in range(s.num_layers)]
        self.v = [self._pool[1, i] for i in range(s.num_layers)]
        self.pool_ptr = self._pool.data_ptr()   # captured decode graphs point here
        self.allocator = BlockAllocator(self.num_blocks)
        self.awake = True

    def sleep(self) -> None:
        self.k, self.v = [], []
        self._pool = None
        self.awake = False

    def copy_block(self, src: int, dst: int) -> None:
        self._pool[:, :, dst].copy_(self._pool[:, :, src])

    def slot(self, block_table: list[int], pos: int) -> int:
        bs = self.spec.block_size
        return block_table[pos // bs] * bs + pos % bs
