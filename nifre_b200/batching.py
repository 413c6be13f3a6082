"""Batch helpers and the cache factory (reference ``src/inference/batching.py:8-55``)."""

from __future__ import annotations

import torch

from .kv_cache import KVCache
from .paged_kv_cache import PagedKVCache


def batch_token_ids(token_lists, device, pad_id):
    """Left-pad token lists to (B, max_len) int64 and return per-row lengths (batching.py:8-19)."""
    width = max(len(t) for t in token_lists)
    rows = [[pad_id] * (width - len(t)) + list(t) for t in token_lists]
    token_ids = torch.tensor(rows, device=device, dtype=torch.long)
    input_lens = torch.tensor([len(t) for t in token_lists], device=device, dtype=torch.long)
    return token_ids, input_lens


def make_kv_cache(model_config, device, dtype=None) -> KVCache:
    """Dense per-row KVCache for a ModelConfig (batching.py:22-32); KV heads are the config's ``kv_heads``."""
    kv_heads = getattr(model_config, "kv_heads", model_config.n_heads)
    return KVCache(num_layers=model_config.num_layers, max_seq_len=model_config.max_seq_len, n_heads=kv_heads,
                   head_dim=model_config.head_dim, device=device, dtype=torch.float16 if dtype is None else dtype)


def make_paged_kv_cache(model_config, device, dtype=None, block_size: int | None = None,
                        enable_prefix_cache: bool = True, prefix_cache_max_entries: int = 1024) -> PagedKVCache:
    """PagedKVCache for a ModelConfig (batching.py:35-55); the KV head count is the config's ``kv_heads``."""
    kv_heads = getattr(model_config, "kv_heads", model_config.n_heads)
    return PagedKVCache(num_layers=model_config.num_layers, max_seq_len=model_config.max_seq_len,
                        n_heads=kv_heads, head_dim=model_config.head_dim, device=device,
                        dtype=torch.float16 if dtype is None else dtype,
                        block_size=block_size or model_config.block_size,
                        enable_prefix_cache=enable_prefix_cache, prefix_cache_max_entries=prefix_cache_max_entries)
