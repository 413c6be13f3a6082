"""nifre_b200: B200-native (sm_100a) ragged continuous-batching attention path for nifre.

Drop-in replacements for nifre's ``Attention`` / ``PagedKVCache`` /
``BlockTable`` / ``BlockAllocator`` / ``PrefixCache`` backed by the CUDA
library ``libnifre_b200.so`` (C ABI in ``include/nifre_b200.h``).
"""

from nifre_b200.attention import Attention, causal_attention
from nifre_b200.block_allocator import BlockAllocator, BlockPoolExhaustedError
from nifre_b200.block_table import BlockTable
from nifre_b200.paged_kv_cache import PagedKVCache, StepPlan
from nifre_b200.prefix_cache import PrefixCache

__all__ = ["Attention", "BlockAllocator", "BlockPoolExhaustedError", "BlockTable", "PagedKVCache",
           "PrefixCache", "StepPlan", "causal_attention"]
