"""Block-chained prefix cache (drop-in for nifre's PrefixCache).

Same keys, order and eviction as jyotilakra92/nifre
``src/inference/prefix_cache.py:14-100``: a prompt's full blocks are keyed by
``(parent_hash, tuple(block_tokens))`` with ``parent_hash = hash((parent,
tokens))`` starting from 0, the longest chain of present keys is the match,
entries live in LRU order with ``max_entries`` and every inserted entry holds
one reference on its block.  The chaining must stay identical: which blocks
are shared -- and therefore the block ids every later allocation returns --
depends on it.
"""

from __future__ import annotations

from collections import OrderedDict

from nifre_b200.block_allocator import BlockAllocator


class PrefixCache:
    ROOT_HASH = 0

    def __init__(self, block_allocator: BlockAllocator, block_size: int, max_entries: int = 1024) -> None:
        if block_size <= 0:
            raise ValueError(f"block_size must be positive, got {block_size}")
        if max_entries <= 0:
            raise ValueError(f"max_entries must be positive, got {max_entries}")
        self.block_allocator = block_allocator
        self.block_size = block_size
        self.max_entries = max_entries
        self.entries: OrderedDict = OrderedDict()
        self.lookups = 0
        self.hits = 0
        self.tokens_saved = 0

    def _blocks_of(self, token_ids):
        bs = self.block_size
        for i in range(len(token_ids) // bs):
            yield i, tuple(token_ids[i * bs:(i + 1) * bs])

    def lookup(self, token_ids: list[int]) -> tuple[int, list[int]]:
        self.lookups += 1
        parent = self.ROOT_HASH
        found: list[int] = []
        for _, blk in self._blocks_of(token_ids):
            key = (parent, blk)
            block_id = self.entries.get(key)
            if block_id is None:
                break
            found.append(block_id)
            self.entries.move_to_end(key)
            parent = self._chain(parent, blk)
        matched = len(found) * self.block_size
        if matched > 0:
            self.hits += 1
            self.tokens_saved += matched
        return matched, found

    def insert(self, token_ids: list[int], physical_blocks: list[int]) -> None:
        parent = self.ROOT_HASH
        for i, blk in self._blocks_of(token_ids):
            if i >= len(physical_blocks):
                break
            key = (parent, blk)
            if key not in self.entries:
                while len(self.entries) >= self.max_entries:
                    self._evict_oldest()
                self.entries[key] = physical_blocks[i]
                self.block_allocator.retain(physical_blocks[i])
            self.entries.move_to_end(key)
            parent = self._chain(parent, blk)

    def _evict_oldest(self) -> None:
        _, block_id = self.entries.popitem(last=False)
        self.block_allocator.release(block_id)

    @staticmethod
    def _chain(parent_hash: int, block_tokens: tuple) -> int:
        return hash((parent_hash, block_tokens))

    def snapshot(self) -> dict:
        rate = self.hits / self.lookups if self.lookups else 0.0
        return {"lookups": self.lookups, "hits": self.hits, "hit_rate": round(rate, 4),
                "tokens_saved": self.tokens_saved, "entries": len(self.entries),
                "max_entries": self.max_entries}
