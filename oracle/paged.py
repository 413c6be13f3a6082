"""CPU restatement of nifre's paged KV storage (oracle; test infrastructure only).

Each class follows one reference file of jyotilakra92/nifre:

* ``OracleAllocator``   -- ``src/inference/block_allocator.py:17-110``
  free list ``list(range(N))`` handed out with ``pop()`` from the end, so the
  first block allocated is ``N-1`` and a freed block is the next one reused
  (``block_allocator.py:57-63,88-92``); refcounts via retain/release.
* ``OracleTable``       -- ``src/inference/block_table.py:13-48``
  ``ensure_capacity`` appends one allocation per missing block, ``resolve`` maps
  token ``t`` to ``(blocks[t // bs], t % bs)``.
* ``OraclePrefixIndex`` -- ``src/inference/prefix_cache.py:14-89``
  chained keys ``(parent_hash, tuple(block_tokens))`` with
  ``parent = hash((parent, tokens))``, LRU order, full blocks only.
* ``OracleStore``       -- ``src/inference/paged_kv_cache.py:51-153``
  per-layer pools ``(num_blocks, bs, H, D)``; ``append`` writes token by token
  through ``resolve`` and advances ``pos`` only on the last layer
  (``paged_kv_cache.py:107-121``); ``get`` concatenates the first ``pos`` rows
  of the slot's blocks (``:123-142``).

The store keeps ``n_heads`` = number of KV heads: the reference has a single
head count, and grouped-query shapes are represented by storing the KV heads
and expanding them at attention time (see ``oracle.attention``).
"""

from __future__ import annotations

from collections import OrderedDict

import torch


class OraclePoolExhausted(RuntimeError):
    pass


class OracleAllocator:
    """block_allocator.py:17-110 restated."""

    def __init__(self, num_blocks: int, free_order: list[int] | None = None):
        self.num_blocks = num_blocks
        # free_order lets a workload start from a permuted free list (the
        # random-permutation block tables of the 1B decode configuration).
        self.free = list(range(num_blocks)) if free_order is None else list(free_order)
        self.refcount = [0] * num_blocks

    def allocate(self) -> int:
        if not self.free:
            raise OraclePoolExhausted("need 1 blocks, only 0 free")
        b = self.free.pop()
        self.refcount[b] = 1
        return b

    def retain(self, b: int) -> None:
        if self.refcount[b] <= 0:
            raise ValueError(f"block {b} is not allocated")
        self.refcount[b] += 1

    def release(self, b: int) -> None:
        if self.refcount[b] <= 0:
            raise ValueError(f"block {b} is not allocated")
        self.refcount[b] -= 1
        if self.refcount[b] == 0:
            self.free.append(b)

    @property
    def allocated(self) -> int:
        return sum(1 for r in self.refcount if r > 0)


class OracleTable:
    """block_table.py:13-48 restated."""

    def __init__(self, alloc: OracleAllocator, block_size: int):
        self.alloc = alloc
        self.bs = block_size
        self.blocks: list[int] = []

    def ensure(self, total_tokens: int) -> None:
        need = (total_tokens + self.bs - 1) // self.bs
        while len(self.blocks) < need:
            self.blocks.append(self.alloc.allocate())

    def resolve(self, t: int) -> tuple[int, int]:
        lb = t // self.bs
        if lb >= len(self.blocks):
            raise IndexError(f"token_index {t} has no allocated block")
        return self.blocks[lb], t % self.bs

    def import_blocks(self, blocks: list[int]) -> None:
        if self.blocks:
            raise ValueError("cannot import blocks into a non-empty block table")
        for b in blocks:
            self.alloc.retain(b)
        self.blocks = list(blocks)

    def clear(self) -> None:
        for b in self.blocks:
            self.alloc.release(b)
        self.blocks = []


class OraclePrefixIndex:
    """prefix_cache.py:14-89 restated (lookup, insert, LRU eviction)."""

    def __init__(self, alloc: OracleAllocator, block_size: int, max_entries: int = 1024):
        self.alloc = alloc
        self.bs = block_size
        self.max_entries = max_entries
        self.entries: OrderedDict = OrderedDict()
        self.lookups = 0
        self.hits = 0
        self.tokens_saved = 0

    def lookup(self, tokens: list[int]) -> tuple[int, list[int]]:
        self.lookups += 1
        parent = 0
        found: list[int] = []
        for i in range(len(tokens) // self.bs):
            blk = tuple(tokens[i * self.bs:(i + 1) * self.bs])
            key = (parent, blk)
            b = self.entries.get(key)
            if b is None:
                break
            found.append(b)
            self.entries.move_to_end(key)
            parent = hash((parent, blk))
        n = len(found) * self.bs
        if n:
            self.hits += 1
            self.tokens_saved += n
        return n, found

    def insert(self, tokens: list[int], blocks: list[int]) -> None:
        parent = 0
        for i in range(len(tokens) // self.bs):
            if i >= len(blocks):
                break
            blk = tuple(tokens[i * self.bs:(i + 1) * self.bs])
            key = (parent, blk)
            if key not in self.entries:
                while len(self.entries) >= self.max_entries:
                    _, old = self.entries.popitem(last=False)
                    self.alloc.release(old)
                self.entries[key] = blocks[i]
                self.alloc.retain(blocks[i])
            self.entries.move_to_end(key)
            parent = hash((parent, blk))


class OracleStore:
    """paged_kv_cache.py:51-153 restated, for ``num_kv_heads`` stored heads."""

    def __init__(self, num_layers: int, max_seq_len: int, num_kv_heads: int, head_dim: int,
                 batch_size: int, dtype: torch.dtype = torch.float32, block_size: int = 16,
                 num_blocks: int | None = None, free_order: list[int] | None = None,
                 prefix: bool = True, prefix_max_entries: int = 1024):
        self.L, self.max_seq_len, self.H, self.D = num_layers, max_seq_len, num_kv_heads, head_dim
        self.bs = block_size
        per_slot = (max_seq_len + block_size - 1) // block_size
        self.num_blocks = per_slot * batch_size if num_blocks is None else num_blocks
        self.alloc = OracleAllocator(self.num_blocks, free_order)
        self.tables = [OracleTable(self.alloc, block_size) for _ in range(batch_size)]
        self.prefix = OraclePrefixIndex(self.alloc, block_size, prefix_max_entries) if prefix else None
        self.pos = [0] * batch_size
        shape = (self.num_blocks, block_size, num_kv_heads, head_dim)
        # zeros instead of the reference's torch.empty: unwritten rows are
        # never read, zeros only make dumps reproducible.
        self.k = [torch.zeros(shape, dtype=dtype) for _ in range(num_layers)]
        self.v = [torch.zeros(shape, dtype=dtype) for _ in range(num_layers)]

    # paged_kv_cache.py:107-121
    def append(self, slot: int, layer: int, key: torch.Tensor, value: torch.Tensor) -> None:
        p = self.pos[slot]
        n = key.shape[0]
        assert p + n <= self.max_seq_len
        tab = self.tables[slot]
        tab.ensure(p + n)
        for i in range(n):
            b, off = tab.resolve(p + i)
            self.k[layer][b, off] = key[i]
            self.v[layer][b, off] = value[i]
        if layer == self.L - 1:
            self.pos[slot] += n

    # paged_kv_cache.py:123-142
    def get(self, slot: int, layer: int) -> tuple[torch.Tensor, torch.Tensor]:
        p = self.pos[slot]
        if p == 0:
            e = torch.empty(0, self.H, self.D, dtype=self.k[layer].dtype)
            return e, e.clone()
        ks, vs, rem = [], [], p
        for b in self.tables[slot].blocks:
            if rem <= 0:
                break
            take = min(rem, self.bs)
            ks.append(self.k[layer][b, :take])
            vs.append(self.v[layer][b, :take])
            rem -= take
        return torch.cat(ks, 0), torch.cat(vs, 0)

    # paged_kv_cache.py:87-105
    def try_load_prefix(self, slot: int, tokens: list[int]) -> int:
        if self.prefix is None:
            return 0
        n, blocks = self.prefix.lookup(tokens)
        if n == 0:
            return 0
        self.tables[slot].import_blocks(blocks)
        self.pos[slot] = n
        return n

    def register_prefix(self, slot: int, tokens: list[int]) -> None:
        if self.prefix is not None:
            self.prefix.insert(tokens, list(self.tables[slot].blocks))

    # paged_kv_cache.py:150-153
    def reset_slot(self, slot: int) -> None:
        self.tables[slot].clear()
        self.pos[slot] = 0

    def slot_of(self, slot: int, t: int) -> int:
        """Flat pool row of token ``t`` of ``slot``: ``block * bs + offset``."""
        b, off = self.tables[slot].resolve(t)
        return b * self.bs + off
