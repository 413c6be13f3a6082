"""Dense per-row KV cache on the paged kernels (drop-in for nifre's KVCache).

Same constructor, attributes and methods as jyotilakra92/nifre
``src/inference/kv_cache.py:4-79``: per layer one ``(batch_size,
max_seq_len, n_heads, head_dim)`` tensor for K and one for V, a write cursor
``pos`` per row that advances after the last layer's append, ``get``
returning views of the first ``pos`` rows, ``reset_slot`` clearing only the
cursor.

That tensor is exactly a paged pool of ``batch_size`` blocks of
``max_seq_len`` tokens with row ``b`` owning block ``b`` (the identity block
table), so the class is a ``PagedKVCache`` whose tables are fixed at
``init_batch``: appends, decode and chunked prefill run through the same
kernels and step plans (``Attention`` accepts either cache), with no prefix
sharing (the reference's dense cache has none).
"""

from __future__ import annotations

import torch

from nifre_b200.paged_kv_cache import PagedKVCache


class KVCache(PagedKVCache):
    def __init__(self, num_layers, max_seq_len, n_heads, head_dim, device="cuda", dtype=torch.float16):
        super().__init__(num_layers, max_seq_len, n_heads, head_dim, device=device, dtype=dtype,
                         block_size=max_seq_len, enable_prefix_cache=False)

    def init_batch(self, batch_size: int) -> None:
        super().init_batch(batch_size)  # batch_size blocks of max_seq_len tokens
        taken = self.block_allocator.allocate_many(batch_size)
        assert sorted(taken) == list(range(batch_size))
        for b, table in enumerate(self.block_tables):
            table.import_blocks([b])  # row b owns block b for the cache's lifetime
        self.block_allocator.free_many(taken)  # the tables hold the only references

    def get(self, batch_idx: int, layer_id: int) -> tuple[torch.Tensor, torch.Tensor]:
        """Views of row ``batch_idx``'s first ``pos`` keys and values (kv_cache.py:66-68)."""
        pos = int(self.pos_host[batch_idx])
        return self.k[layer_id][batch_idx, :pos], self.v[layer_id][batch_idx, :pos]

    def reset_slot(self, batch_idx: int) -> None:
        """Clear the row's write cursor; the row keeps its storage (kv_cache.py:75-77)."""
        self._set_pos(batch_idx, 0)
