"""Per-sequence logical -> physical block map (drop-in for nifre's BlockTable).

Semantics of jyotilakra92/nifre ``src/inference/block_table.py:3-48``:
``ensure_capacity`` appends one allocation per missing block, ``resolve`` maps
token ``t`` to ``(blocks[t // bs], t % bs)`` and raises IndexError past the
allocated blocks, ``import_blocks`` attaches (and retains) shared prefix blocks
to an empty table, ``clear`` releases every reference.

The host table is the authority; the cache mirrors it into a device tensor.
``epoch`` changes whenever existing entries are replaced (clear/import), so
the mirror knows when it must rewrite a row rather than append to it.
"""

from __future__ import annotations

from nifre_b200.block_allocator import BlockAllocator, BlockPoolExhaustedError


class BlockTable:
    def __init__(self, allocator: BlockAllocator, block_size: int) -> None:
        if block_size <= 0:
            raise ValueError(f"block_size must be positive, got {block_size}")
        self._allocator = allocator
        self._block_size = block_size
        self._physical_blocks: list[int] = []
        self.epoch = 0

    def import_blocks(self, physical_blocks: list[int]) -> None:
        if self._physical_blocks:
            raise ValueError("cannot import blocks into a non-empty block table")
        for block_id in physical_blocks:
            self._allocator.retain(block_id)
        self._physical_blocks = list(physical_blocks)
        self.epoch += 1

    def ensure_capacity(self, total_tokens: int) -> None:
        if total_tokens < 0:
            raise ValueError(f"total_tokens must be non-negative, got {total_tokens}")
        need = (total_tokens + self._block_size - 1) // self._block_size - len(self._physical_blocks)
        if need <= 0:
            return
        avail = self._allocator.free_count
        if need <= avail:
            self._physical_blocks.extend(self._allocator.allocate_many(need))
            return
        # the reference allocates one block at a time: take what is left, then fail
        if avail:
            self._physical_blocks.extend(self._allocator.allocate_many(avail))
        raise BlockPoolExhaustedError("need 1 blocks, only 0 free")

    def resolve(self, token_index: int) -> tuple[int, int]:
        logical = token_index // self._block_size
        if logical >= len(self._physical_blocks):
            raise IndexError(f"token_index {token_index} has no allocated block")
        return self._physical_blocks[logical], token_index % self._block_size

    def physical_blocks(self) -> list[int]:
        return self._physical_blocks[:]

    def __len__(self) -> int:
        return len(self._physical_blocks)

    def clear(self) -> None:
        if self._physical_blocks:
            self._allocator.free_many(self._physical_blocks)
            self._physical_blocks.clear()
        self.epoch += 1
