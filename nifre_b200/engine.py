"""Continuous-batching engine: scheduler + model runner + paged KV cache.

Public behaviour of the reference's ``src/inference/engine.py:21-288``
(``add_request``, ``step``, ``run_until_done``, ``generate``,
``generate_stream``, ``get_completed``, ``get_config``, ``reconfigure``, token
callbacks, metrics hooks).  A step schedules, runs the prefill chunks, then
the decodes, and applies the same bookkeeping in the same order: prefix
registration of completed prompts, the first token, slot release of finished
requests (``engine.py:243-288``).

B200 difference: when nothing between the reference's prefill forward and its
decode forward can change the block allocator (no request finishes at its
first token, so no slot is reset; no prefix registration can evict), the
prefill chunks and the decodes run as ONE forward with prefill rows first —
the allocation order the reference's two forwards produce.  Otherwise the
step runs the two forwards like the reference.
"""

from __future__ import annotations

import time
import uuid
from queue import Empty, Queue
from typing import Callable, Iterator, List, Optional

import torch

from .batching import make_kv_cache, make_paged_kv_cache
from .data_model import EngineConfig, InferenceRequest, RequestState, validate_engine_config
from .model_runner import ModelRunner
from .scheduler import Scheduler

TokenCallback = Callable[[int], None]


class Engine:
    def __init__(self, model, max_concurrent_requests: int, device, metrics_collector=None,
                 prefill_chunk_size: int = 128, max_tokens_per_step: int = 2048, use_paged_kv_cache: bool = True,
                 use_prefix_cache: bool = True, use_cuda_graphs: bool = True):
        self.model = model
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("nifre_b200.Engine runs on a CUDA device")
        self.max_concurrent_requests = max_concurrent_requests
        self.scheduler = Scheduler(max_concurrent_requests, max_tokens_per_step)
        self.model_runner = ModelRunner(model, self.device, use_cuda_graphs=use_cuda_graphs)
        self.cache = None
        self.metrics = metrics_collector
        self.prefill_chunk_size = prefill_chunk_size
        self.max_tokens_per_step = max_tokens_per_step
        if getattr(model, "supports_prefix_cache", True) is False:
            use_prefix_cache = False
        self.use_paged_kv_cache = use_paged_kv_cache
        self.use_prefix_cache = use_prefix_cache
        self._token_callbacks: dict[str, TokenCallback] = {}
        self.steps = 0
        self.fused_steps = 0

    # ------------------------------------------------------------------ requests
    def add_request(self, prompt_token_ids: List[int], max_new_tokens: int) -> str:
        request_id = uuid.uuid4().hex[:8]
        self.scheduler.add_request(InferenceRequest(request_id=request_id, prompt_token_ids=list(prompt_token_ids),
                                                    max_new_tokens=max_new_tokens,
                                                    prefill_chunk_size=self.prefill_chunk_size))
        if self.metrics:
            self.metrics.on_request_enqueued()
        return request_id

    def get_completed(self) -> dict:
        return self.scheduler.completed

    def register_token_callback(self, request_id: str, callback: TokenCallback) -> None:
        self._token_callbacks[request_id] = callback

    def unregister_token_callback(self, request_id: str) -> None:
        self._token_callbacks.pop(request_id, None)

    def _emit(self, request_id: str, token_id: int) -> None:
        callback = self._token_callbacks.get(request_id)
        if callback is not None:
            callback(token_id)

    # ------------------------------------------------------------------ stepping
    def _ensure_cache(self) -> None:
        if self.cache is not None:
            return
        make = getattr(self.model, "make_kv_cache", None)
        dtype = getattr(self.model, "dtype", torch.float16)
        if make is not None:
            self.cache = make(self.device, enable_prefix_cache=self.use_prefix_cache)
        elif self.use_paged_kv_cache:
            self.cache = make_paged_kv_cache(self.model.config, self.device, dtype=dtype,
                                             enable_prefix_cache=self.use_prefix_cache)
        else:  # engine.py:226-227: the dense per-row cache
            self.cache = make_kv_cache(self.model.config, self.device, dtype=dtype)
        self.cache.init_batch(self.max_concurrent_requests)

    def _fusable(self, prefills: List[InferenceRequest]) -> bool:
        """True when the prefill half of the step cannot free or evict blocks before the decodes allocate."""
        pc = getattr(self.cache, "prefix_cache", None)
        new_keys = 0
        for request in prefills:
            if request.next_chunk()[1] < request.num_prompt_tokens:
                continue
            if request.num_generated + 1 >= request.max_new_tokens:
                return False  # finishes at its first token: its slot is reset before the decodes
            new_keys += request.num_prompt_tokens // self.cache.block_size
        return pc is None or len(pc.entries) + new_keys <= pc.max_entries

    def step(self) -> bool:
        if not self.scheduler.has_work():
            return False
        self._ensure_cache()
        result = self.scheduler.schedule()
        prefills, decodes = result.prefill_requests, result.decode_requests
        self.steps += 1
        if prefills and decodes and self.model_runner.flat:
            ModelRunner.prepare(self.cache, prefills)
            if self._fusable(prefills):
                self.fused_steps += 1
                processed = self._chunk_tokens(prefills)
                t0 = time.perf_counter()
                pre, dec = self.model_runner.run_step(self.cache, prefills, decodes)
                dt = time.perf_counter() - t0
                self._after_prefill(prefills, pre, dt, processed)
                self._after_decode(decodes, dec, dt)
                return True
        if prefills:
            processed = self._chunk_tokens(prefills)
            t0 = time.perf_counter()
            pre, _ = self.model_runner.run_step(self.cache, prefills, [])
            self._after_prefill(prefills, pre, time.perf_counter() - t0, processed)
        if decodes:
            t0 = time.perf_counter()
            _, dec = self.model_runner.run_step(self.cache, [], decodes)
            self._after_decode(decodes, dec, time.perf_counter() - t0)
        return True

    @staticmethod
    def _chunk_tokens(requests) -> int:
        return sum(end - start for start, end in (r.next_chunk() for r in requests))

    def _after_prefill(self, requests, tokens, duration, processed) -> None:
        if self.metrics:
            for request in requests:
                if request.prefix_cache_hit_tokens > 0:
                    self.metrics.on_prefix_cache_hit(request.prefix_cache_hit_tokens)
            self.metrics.on_prefill_batch(requests, duration, processed)
        for request, token in zip(requests, tokens):
            if request.prefill_complete and hasattr(self.cache, "register_prefix"):
                self.cache.register_prefix(request.batch_idx, request.prompt_token_ids)
            if token is None:
                continue
            slot = request.batch_idx
            self.scheduler.mark_prefill_done(request)
            self.scheduler.mark_decode_done(request, token)
            self._emit(request.request_id, token)
            if self.metrics and request.state == RequestState.FINISHED:
                self.metrics.on_request_finished(request)
            self._release(slot, request)

    def _after_decode(self, requests, tokens, duration) -> None:
        if self.metrics:
            self.metrics.on_decode_batch(len(requests), duration)
        for request, token in zip(requests, tokens):
            slot = request.batch_idx
            self.scheduler.mark_decode_done(request, token)
            self._emit(request.request_id, token)
            if self.metrics:
                self.metrics.on_decode_token(request)
                if request.state == RequestState.FINISHED:
                    self.metrics.on_request_finished(request)
            self._release(slot, request)

    def _release(self, slot: Optional[int], request: InferenceRequest) -> None:
        if request.state == RequestState.FINISHED and self.cache is not None and slot is not None:
            self.cache.reset_slot(slot)

    def run_until_done(self) -> None:
        while self.step():
            pass

    # ------------------------------------------------------------------ convenience
    def generate(self, prompt_token_ids: List[int], max_new_tokens: int,
                 timeout_seconds: Optional[float] = None) -> InferenceRequest:
        request_id = self.add_request(prompt_token_ids, max_new_tokens)
        deadline = time.time() + timeout_seconds if timeout_seconds else None
        try:
            while request_id not in self.scheduler.completed and request_id not in self.scheduler.failed:
                if deadline and time.time() > deadline:
                    request = self._cancel(request_id, "timeout")
                    if self.metrics and request is not None:
                        self.metrics.on_request_failed(request, "timeout")
                    return self.scheduler.failed[request_id]
                self.step()
        finally:
            self.unregister_token_callback(request_id)
        return self.scheduler.completed.get(request_id) or self.scheduler.failed[request_id]

    def generate_stream(self, prompt_token_ids: List[int], max_new_tokens: int) -> Iterator[int]:
        request_id = self.add_request(prompt_token_ids, max_new_tokens)
        queue: Queue = Queue()
        self.register_token_callback(request_id, queue.put)
        try:
            while request_id not in self.scheduler.completed and request_id not in self.scheduler.failed:
                self.step()
                while True:
                    try:
                        yield queue.get_nowait()
                    except Empty:
                        break
        finally:
            self.unregister_token_callback(request_id)

    def _cancel(self, request_id: str, status: str) -> Optional[InferenceRequest]:
        # As in engine.py:196-200 the slot is not reset here (the scheduler has
        # already cleared batch_idx); its blocks are freed when the slot is next
        # prepared, which keeps block ids identical to the reference's.
        return self.scheduler.cancel_request(request_id, status=status)

    def get_config(self) -> EngineConfig:
        return EngineConfig(max_concurrent_requests=self.max_concurrent_requests,
                            prefill_chunk_size=self.prefill_chunk_size,
                            max_tokens_per_step=self.max_tokens_per_step,
                            use_paged_kv_cache=self.use_paged_kv_cache, use_prefix_cache=self.use_prefix_cache)

    def reconfigure(self, *, prefill_chunk_size: int | None = None, max_tokens_per_step: int | None = None,
                    max_concurrent_requests: int | None = None, use_paged_kv_cache: bool | None = None,
                    use_prefix_cache: bool | None = None) -> EngineConfig:
        validate_engine_config(max_concurrent_requests=max_concurrent_requests,
                               prefill_chunk_size=prefill_chunk_size, max_tokens_per_step=max_tokens_per_step)
        built = self.cache is not None
        if use_paged_kv_cache is not None and use_paged_kv_cache != self.use_paged_kv_cache:
            if built:
                raise ValueError("cannot change use_paged_kv_cache after KV cache is initialized")
            self.use_paged_kv_cache = use_paged_kv_cache
        if use_prefix_cache is not None and use_prefix_cache != self.use_prefix_cache:
            if built:
                raise ValueError("cannot change use_prefix_cache after KV cache is initialized")
            self.use_prefix_cache = use_prefix_cache
        if prefill_chunk_size is not None:
            self.prefill_chunk_size = prefill_chunk_size
        if max_tokens_per_step is not None:
            self.max_tokens_per_step = max_tokens_per_step
        if max_tokens_per_step is not None or max_concurrent_requests is not None:
            self.scheduler.reconfigure(max_tokens_per_step=max_tokens_per_step,
                                       max_concurrent_requests=max_concurrent_requests, cache_initialized=built)
            if max_concurrent_requests is not None:
                self.max_concurrent_requests = max_concurrent_requests
        return self.get_config()
