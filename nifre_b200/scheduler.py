"""Continuous-batching scheduler (host).

Behaviour of the reference's ``src/inference/scheduler.py:7-180``, which
decides which rows exist in a step and therefore the block-allocation order
the KV cache must reproduce bit for bit:

* waiting requests take free slots FIFO, the lowest free slot first as the
  slots were freed (``_assign_waiting_to_slots``, ``:139-145``);
* decode requests come first, one token each, in ``running`` insertion order,
  until the token budget is spent (``:32-41``);
* then every PREFILL request whose next chunk ``min(chunk, remaining)`` fits
  the remaining budget, skipping (not stopping at) those that do not
  (``:43-49``);
* finishing a request returns its slot to the end of the free list
  (``:170-176``).
"""

from __future__ import annotations

from collections import deque

from .data_model import InferenceRequest, RequestState, ScheduleResult


def _positive(name: str, value: int) -> None:
    if value <= 0:
        raise ValueError(f"{name} must be positive, got {value}")


class Scheduler:
    def __init__(self, max_concurrent_requests: int, max_tokens_per_step: int = 2048):
        _positive("max_concurrent_requests", max_concurrent_requests)
        _positive("max_tokens_per_step", max_tokens_per_step)
        self.max_concurrent_requests = max_concurrent_requests
        self.max_tokens_per_step = max_tokens_per_step
        self.waiting: deque = deque()
        self.running: dict = {}
        self.completed: dict = {}
        self.failed: dict = {}
        self.free_slots: list = list(range(max_concurrent_requests))

    # ------------------------------------------------------------------ queueing
    def add_request(self, request: InferenceRequest) -> None:
        if request.state != RequestState.WAITING:
            raise ValueError("new requests must start in WAITING")
        self.waiting.append(request)

    def has_work(self) -> bool:
        return bool(self.waiting) or bool(self.running)

    def _admit(self) -> None:
        while self.waiting and self.free_slots:
            request = self.waiting.popleft()
            request.batch_idx = self.free_slots.pop(0)
            request.state = RequestState.PREFILL
            self.running[request.request_id] = request

    @staticmethod
    def _chunk_tokens(request: InferenceRequest) -> int:
        return min(request.prefill_chunk_size, request.num_prompt_tokens - request.prefill_offset)

    def schedule(self) -> ScheduleResult:
        self._admit()
        budget = self.max_tokens_per_step
        decodes = []
        for request in self.running.values():
            if request.state is not RequestState.DECODE:
                continue
            if budget < 1:
                break
            decodes.append(request)
            budget -= 1
        prefills = []
        for request in self.running.values():
            if request.state is not RequestState.PREFILL:
                continue
            need = self._chunk_tokens(request)
            if need <= budget:
                prefills.append(request)
                budget -= need
        return ScheduleResult(prefill_requests=prefills, decode_requests=decodes)

    # ------------------------------------------------------------------ transitions
    def mark_prefill_done(self, request: InferenceRequest) -> None:
        if request.state != RequestState.PREFILL:
            raise ValueError(f"expected PREFILL, got {request.state}")
        if not request.prefill_complete:
            raise ValueError(f"prefill incomplete: offset={request.prefill_offset}, "
                             f"prompt_len={request.num_prompt_tokens}")
        request.state = RequestState.DECODE

    def mark_decode_done(self, request: InferenceRequest, token_id: int) -> None:
        if request.state != RequestState.DECODE:
            raise ValueError(f"expected DECODE, got {request.state}")
        request.output_token_ids.append(token_id)
        if request.num_generated >= request.max_new_tokens:
            request.state = RequestState.FINISHED
            del self.running[request.request_id]
            self.completed[request.request_id] = request
            self._release(request)

    def _release(self, request: InferenceRequest) -> None:
        if request.batch_idx is not None:
            self.free_slots.append(request.batch_idx)
            request.batch_idx = None

    def cancel_request(self, request_id: str, status: str = "timeout") -> InferenceRequest:
        """Drop a waiting or running request and record it as failed."""
        for request in self.waiting:
            if request.request_id == request_id:
                self.waiting = deque(r for r in self.waiting if r.request_id != request_id)
                request.state = RequestState.FINISHED
                request.status = status
                self.failed[request_id] = request
                return request
        request = self.running.pop(request_id, None)
        if request is None:
            raise KeyError(f"unknown request_id: {request_id}")
        request.state = RequestState.FINISHED
        request.status = status
        self._release(request)
        self.failed[request_id] = request
        return request

    # ------------------------------------------------------------------ runtime settings
    def reconfigure(self, *, max_tokens_per_step: int | None = None, max_concurrent_requests: int | None = None,
                    cache_initialized: bool = False) -> None:
        if max_tokens_per_step is not None:
            _positive("max_tokens_per_step", max_tokens_per_step)
            self.max_tokens_per_step = max_tokens_per_step
        if max_concurrent_requests is not None:
            self._resize(max_concurrent_requests, cache_initialized)

    def _resize(self, new_max: int, cache_initialized: bool) -> None:
        _positive("max_concurrent_requests", new_max)
        old = self.max_concurrent_requests
        if new_max == old:
            return
        if cache_initialized and new_max > old:
            raise ValueError("cannot increase max_concurrent_requests after KV cache is initialized")
        if len(self.running) > new_max:
            raise ValueError(f"cannot set max_concurrent_requests to {new_max} with "
                             f"{len(self.running)} running requests")
        for request in self.running.values():
            if request.batch_idx is not None and request.batch_idx >= new_max:
                raise ValueError(f"running request uses slot {request.batch_idx}, above new max {new_max}")
        if new_max > old:
            self.free_slots.extend(s for s in range(old, new_max) if s not in self.free_slots)
        else:
            self.free_slots = [s for s in self.free_slots if s < new_max]
        self.free_slots.sort()
        self.max_concurrent_requests = new_max
