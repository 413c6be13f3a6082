"""Host-side pool of physical KV block ids (drop-in for nifre's BlockAllocator).

Same public API, allocation order and errors as the reference
(jyotilakra92/nifre ``src/inference/block_allocator.py:10-116``): the free
ids form a stack that starts as ``0..N-1`` and is popped from the top, so the
first id handed out is ``N-1`` and a freed id is the next one reused
(``:57-63``, ``:88-92``); refcounts back shared prefix blocks (``:65-82``).

The state lives in numpy arrays so that a step's allocations for a long
prefill chunk (dozens of blocks) are one slice, not a Python loop; the ids
produced are identical to the reference's one-at-a-time ``pop()``.
"""

from __future__ import annotations

import numpy as np


class BlockPoolExhaustedError(RuntimeError):
    """Raised when the KV block pool has no free blocks left."""


class BlockAllocator:
    def __init__(self, num_blocks: int) -> None:
        if num_blocks <= 0:
            raise ValueError(f"num_blocks must be positive, got {num_blocks}")
        self._num_blocks = int(num_blocks)
        self._stack = np.arange(self._num_blocks, dtype=np.int64)  # free ids, top = end
        self._top = self._num_blocks
        self._refcount = np.zeros(self._num_blocks, dtype=np.int64)
        self._allocated = 0

    # ---------------------------------------------------------------- queries
    @property
    def num_blocks(self) -> int:
        return self._num_blocks

    @property
    def allocated_count(self) -> int:
        return self._allocated

    @property
    def free_count(self) -> int:
        return self._top

    @property
    def utilization(self) -> float:
        return self._allocated / self._num_blocks

    def free_ids(self) -> list[int]:
        """Free ids bottom-to-top (the next allocation is the last element)."""
        return self._stack[: self._top].tolist()

    def set_free_order(self, ids) -> None:
        """Replace the free stack of a pool with no live blocks (bottom-to-top order).

        Used to start from a permuted pool, the way a long-running server's free
        list ends up shuffled.
        """
        ids = np.asarray(ids, dtype=np.int64)
        if self._allocated:
            raise ValueError("set_free_order needs a pool with no allocated blocks")
        if ids.shape != (self._num_blocks,) or not np.array_equal(np.sort(ids), np.arange(self._num_blocks)):
            raise ValueError("set_free_order needs a permutation of all block ids")
        self._stack[:] = ids
        self._top = self._num_blocks

    # ---------------------------------------------------------------- allocation
    def allocate(self) -> int:
        """Allocate one block. Prefer `allocate_many` for multiple blocks."""
        return self.allocate_many(1)[0]

    def allocate_many(self, count: int) -> list[int]:
        if count <= 0:
            raise ValueError(f"count must be positive, got {count}")
        if count > self._top:
            raise BlockPoolExhaustedError(f"need {count} blocks, only {self._top} free")
        ids = self._stack[self._top - count: self._top][::-1].copy()
        self._top -= count
        self._refcount[ids] = 1
        self._allocated += count
        return ids.tolist()

    def retain(self, block_id: int) -> None:
        self._validate_block_id(block_id)
        if self._refcount[block_id] <= 0:
            raise ValueError(f"block {block_id} is not allocated")
        self._refcount[block_id] += 1

    def release(self, block_id: int) -> None:
        self._validate_block_id(block_id)
        if self._refcount[block_id] <= 0:
            raise ValueError(f"block {block_id} is not allocated")
        self._refcount[block_id] -= 1
        if self._refcount[block_id] == 0:
            self._stack[self._top] = block_id
            self._top += 1
            self._allocated -= 1

    def refcount(self, block_id: int) -> int:
        self._validate_block_id(block_id)
        return int(self._refcount[block_id])

    def free(self, block_id: int) -> None:
        self.free_many([block_id])

    def free_many(self, block_ids: list[int]) -> None:
        if not block_ids:
            return
        seen: set[int] = set()
        for block_id in block_ids:
            self._validate_block_id(block_id)
            if block_id in seen:
                raise ValueError(f"duplicate block_id in free_many: {block_id}")
            seen.add(block_id)
        for block_id in block_ids:
            self.release(block_id)

    def _validate_block_id(self, block_id: int) -> None:
        if block_id < 0 or block_id >= self._num_blocks:
            raise ValueError(f"block_id {block_id} out of range [0, {self._num_blocks})")

    def __repr__(self) -> str:
        return (f"BlockAllocator(blocks={self._num_blocks}, "
                f"allocated={self.allocated_count}, free={self.free_count})")
