"""nifre_b200: B200-native (sm_100a) ragged continuous-batching attention path for nifre.

Drop-in replacements for nifre's ``Attention`` / ``PagedKVCache`` / ``KVCache`` /
``BlockTable`` / ``BlockAllocator`` / ``PrefixCache`` backed by the CUDA
library ``libnifre_b200.so`` (C ABI in ``include/nifre_b200.h``), and the
engine layer that drives them a whole step at a time (``Engine``,
``Scheduler``, ``ModelRunner``, ``GptModel``).
"""

from nifre_b200.attention import Attention, causal_attention
from nifre_b200.block_allocator import BlockAllocator, BlockPoolExhaustedError
from nifre_b200.block_table import BlockTable
from nifre_b200.kv_cache import KVCache
from nifre_b200.paged_kv_cache import PagedKVCache, StepPlan
from nifre_b200.data_model import (EngineConfig, InferenceRequest, ModelConfig, RequestState, ScheduleResult,
                                   validate_engine_config)
from nifre_b200.engine import Engine
from nifre_b200.gpt import GPT_CONFIG_124M, GptInferenceModel, GptModel
from nifre_b200.model_runner import ModelRunner
from nifre_b200.prefix_cache import PrefixCache
from nifre_b200.scheduler import Scheduler

__all__ = ["Attention", "BlockAllocator", "BlockPoolExhaustedError", "BlockTable", "Engine", "EngineConfig",
           "GPT_CONFIG_124M", "GptInferenceModel", "GptModel", "InferenceRequest", "KVCache", "ModelConfig",
           "ModelRunner", "PagedKVCache", "PrefixCache", "RequestState", "ScheduleResult", "Scheduler", "StepPlan",
           "causal_attention", "validate_engine_config"]
