"""Request, schedule and configuration records of the inference engine.

Same fields, defaults and meaning as the reference's
``src/inference/data_model.py:7-91`` (``RequestState``, ``InferenceRequest``,
``ScheduleResult``, ``ModelConfig``, ``EngineConfig``,
``validate_engine_config``), so engine callers and the scheduler read the same
attributes.  ``ModelConfig`` gains an optional ``num_kv_heads`` (grouped-query
models); ``None`` means ``n_heads``, the reference's only case.
"""

from __future__ import annotations

import time
from dataclasses import dataclass, field
from enum import Enum
from typing import Optional


class RequestState(Enum):
    WAITING = "waiting"
    PREFILL = "prefill"
    DECODE = "decode"
    FINISHED = "finished"


@dataclass
class InferenceRequest:
    request_id: str
    prompt_token_ids: list
    max_new_tokens: int
    state: RequestState = RequestState.WAITING
    output_token_ids: list = field(default_factory=list)
    batch_idx: Optional[int] = None
    created_at: float = field(default_factory=time.time)
    first_token_at: Optional[float] = None
    finished_at: Optional[float] = None
    last_token_at: Optional[float] = None
    prefill_duration_sec: Optional[float] = None
    prefill_offset: int = 0
    prefill_chunk_size: int = 128
    slot_prepared: bool = False
    prefix_cache_hit_tokens: int = 0
    status: str = "ok"

    @property
    def num_prompt_tokens(self) -> int:
        return len(self.prompt_token_ids)

    @property
    def num_generated(self) -> int:
        return len(self.output_token_ids)

    @property
    def prefill_complete(self) -> bool:
        return self.prefill_offset >= self.num_prompt_tokens

    def next_chunk(self) -> tuple[int, int]:
        """Prompt range [start, end) of this request's next prefill chunk."""
        start = self.prefill_offset
        return start, min(start + self.prefill_chunk_size, self.num_prompt_tokens)


@dataclass
class ScheduleResult:
    prefill_requests: list
    decode_requests: list


@dataclass(frozen=True)
class ModelConfig:
    num_layers: int
    max_seq_len: int
    n_heads: int
    head_dim: int
    vocab_size: int
    pad_token_id: int
    block_size: int = 16
    num_kv_heads: Optional[int] = None

    @property
    def kv_heads(self) -> int:
        return self.n_heads if self.num_kv_heads is None else self.num_kv_heads


@dataclass(frozen=True)
class EngineConfig:
    max_concurrent_requests: int
    prefill_chunk_size: int
    max_tokens_per_step: int
    use_paged_kv_cache: bool
    use_prefix_cache: bool


def validate_engine_config(*, max_concurrent_requests: int | None = None, prefill_chunk_size: int | None = None,
                           max_tokens_per_step: int | None = None) -> None:
    """Raise ValueError for a non-positive setting (data_model.py:77-91)."""
    for name, value in (("max_concurrent_requests", max_concurrent_requests),
                        ("prefill_chunk_size", prefill_chunk_size),
                        ("max_tokens_per_step", max_tokens_per_step)):
        if value is not None and value <= 0:
            raise ValueError(f"{name} must be positive, got {value}")
