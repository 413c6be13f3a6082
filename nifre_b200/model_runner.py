"""Forward passes of the engine's steps (host orchestration).

Behaviour of the reference's ``src/inference/model_runner.py:10-86``: slot
preparation on a request's first prefill (prefix-cache import, else a slot
reset), chunk selection from ``prefill_offset``, ``prefill_offset`` advanced by
the chunk, a greedy token when the prompt completes, and the last output token
as the decode input.  The difference is the batch: ``run_step`` runs the
step's prefill chunks and decodes as one flat set of rows through the model's
``forward_step`` (no padding, logits only for sampled rows, argmax on the
device and a single device-to-host copy of the sampled ids).  Models without
``forward_step`` are driven through the reference's padded-batch protocol.

Decode-only steps of a batch repeat the same kernels with the same sizes, so
the runner captures one such step's forward (every layer's projections,
KV append, attention and MLP, the head and the argmax) in a CUDA graph and
replays it while the batch and its plan layout (``StepPlan.layout_key``)
stay the same: per step the host then plans (one upload, one pack launch),
copies the step's ids and positions into the graph's input buffer, launches
the graph and reads the tokens back.
"""

from __future__ import annotations

from typing import List, Optional

import numpy as np
import torch

from .batching import batch_token_ids
from .data_model import InferenceRequest


class ModelRunner:
    def __init__(self, model, device, use_cuda_graphs: bool = True):
        self.model = model
        self.device = torch.device(device)
        self.model.eval()
        self.use_cuda_graphs = use_cuda_graphs
        self._graph = None  # the captured decode step: key, graph, input buffer, tokens, kept buffers
        self._last_key = None  # layout of the previous decode step (a layout is captured when it repeats)
        self.graph_replays = 0

    @property
    def flat(self) -> bool:
        return hasattr(self.model, "forward_step")

    @staticmethod
    def prepare(cache, requests: List[InferenceRequest]) -> None:
        """First-prefill slot preparation (model_runner.py:27-37)."""
        for request in requests:
            if request.slot_prepared:
                continue
            loaded = cache.try_load_prefix(request.batch_idx, request.prompt_token_ids) \
                if hasattr(cache, "try_load_prefix") else 0
            if loaded > 0:
                request.prefill_offset = loaded
                request.prefix_cache_hit_tokens = loaded
            elif request.prefill_offset == 0:
                cache.reset_slot(request.batch_idx)
            request.slot_prepared = True

    @torch.no_grad()
    def run_step(self, cache, prefills: List[InferenceRequest],
                 decodes: List[InferenceRequest]) -> tuple[List[Optional[int]], List[int]]:
        """One forward over the prefill chunks (first, in order) and the decodes.

        Returns the greedy token of each prefill request whose prompt completes
        (else None) and of each decode request.
        """
        self.prepare(cache, prefills)
        if not self.flat:
            pre = self._padded_prefill(cache, prefills) if prefills else []
            dec = self._padded_decode(cache, decodes) if decodes else []
            return pre, dec
        ids: list = []
        lens: list = []
        sample: list = []
        completes: list = []
        for request in prefills:
            start, end = request.next_chunk()
            ids.extend(request.prompt_token_ids[start:end])
            lens.append(end - start)
            completes.append(end >= request.num_prompt_tokens)
            if completes[-1]:
                sample.append(len(ids) - 1)
        for request in decodes:
            ids.append(request.output_token_ids[-1])
            lens.append(1)
            sample.append(len(ids) - 1)
        rows = prefills + decodes
        slots = [r.batch_idx for r in rows]
        starts = np.concatenate([[0], np.cumsum(lens)[:-1]]).astype(np.int64)
        pos0 = cache.pos_host[slots]
        positions = np.repeat(pos0 - starts, lens) + np.arange(len(ids))
        graphed = self.use_cuda_graphs and not prefills and self.device.type == "cuda"
        plan = cache.plan(slots, lens, starts.tolist(), q_heads=getattr(self.model.config, "n_heads", None),
                          fixed_layout=graphed)
        dev = self.device
        host = torch.from_numpy(np.concatenate([np.asarray(ids, np.int64), positions.astype(np.int64),
                                                np.asarray(sample, np.int64)])).pin_memory()
        T, S = len(ids), len(sample)
        if graphed:
            return [], self._graph_decode(cache, plan, host, T, S)
        buf = host.to(dev, non_blocking=True)
        tokens: list = []
        if S:
            logits = self.model.forward_step(buf[:T], buf[T:2 * T], cache, plan, buf[2 * T:2 * T + S])
            tokens = logits.argmax(dim=-1).cpu().tolist()
        else:
            self.model.forward_step(buf[:T], buf[T:2 * T], cache, plan, buf[2 * T:2 * T])
        it = iter(tokens)
        pre: List[Optional[int]] = []
        for request, n, done in zip(prefills, lens, completes):
            request.prefill_offset += n
            pre.append(next(it) if done else None)
        dec = [next(it) for _ in decodes]
        return pre, dec

    def _graph_decode(self, cache, plan, host: torch.Tensor, T: int, S: int) -> List[int]:
        """Greedy tokens of a decode-only step, by replaying (or first capturing) the step's CUDA graph."""
        key = (id(cache), cache.k[0].data_ptr(), plan.layout_key)
        g = self._graph
        if g is not None and g["key"] == key:
            g["inputs"].copy_(host, non_blocking=True)
            g["graph"].replay()
            cache._close(plan)  # the host bookkeeping the captured forward did when it ran
            self.graph_replays += 1
            return g["tokens"].cpu().tolist()
        seen, self._last_key = self._last_key == key, key
        if not seen:  # a new layout runs eagerly once (and warms the libraries up for its sizes)
            return self._eager(cache, plan, host, T, S)
        self._graph = None
        inputs = torch.empty(2 * T + S, dtype=torch.int64, device=self.device)
        inputs.copy_(host, non_blocking=True)
        graph = torch.cuda.CUDAGraph()
        try:
            with torch.cuda.graph(graph):
                logits = self.model.forward_step(inputs[:T], inputs[T:2 * T], cache, plan, inputs[2 * T:])
                tokens = logits.argmax(dim=-1)
        except RuntimeError:
            # capture refused (a launch this driver cannot record): no graphs from here on; the step
            # runs eagerly on the same plan, reopened if the capture had already closed it
            self.use_cuda_graphs = False
            torch.cuda.synchronize(self.device)
            if plan.closed:
                cache.pos_host[plan.slots] = plan.ctx_before
                plan.closed = False
                cache._plan = plan
            return self._eager(cache, plan, host, T, S)
        # the graph reads the plan's metadata buffer and the split-K workspace it was captured with: keep them
        refs = (plan.items, cache._ws_partials.t, cache._ws_counters.t)
        self._graph = dict(key=key, graph=graph, inputs=inputs, tokens=tokens, refs=refs)
        graph.replay()  # capture launched nothing: run this step
        return tokens.cpu().tolist()

    def _eager(self, cache, plan, host: torch.Tensor, T: int, S: int) -> List[int]:
        buf = host.to(self.device, non_blocking=True)
        logits = self.model.forward_step(buf[:T], buf[T:2 * T], cache, plan, buf[2 * T:2 * T + S])
        return logits.argmax(dim=-1).cpu().tolist()

    # ------------------------------------------------------------------ reference protocol
    @torch.no_grad()
    def prefill(self, cache, requests: List[InferenceRequest]) -> List[Optional[int]]:
        return self.run_step(cache, requests, [])[0]

    @torch.no_grad()
    def decode(self, cache, requests: List[InferenceRequest]) -> List[int]:
        return self.run_step(cache, [], requests)[1]

    def _padded_prefill(self, cache, requests):
        chunks = [r.prompt_token_ids[slice(*r.next_chunk())] for r in requests]
        token_ids, input_lens = batch_token_ids(chunks, self.device, pad_id=self.model.config.pad_token_id)
        logits = self.model(token_ids, kv_cache=cache, input_lens=input_lens,
                            cache_batch_indices=[r.batch_idx for r in requests])
        out: List[Optional[int]] = []
        for i, request in enumerate(requests):
            request.prefill_offset += len(chunks[i])
            out.append(int(logits[i, -1].argmax()) if request.prefill_complete else None)
        return out

    def _padded_decode(self, cache, requests):
        token_ids = torch.tensor([[r.output_token_ids[-1]] for r in requests], device=self.device, dtype=torch.long)
        logits = self.model(token_ids, kv_cache=cache, cache_batch_indices=[r.batch_idx for r in requests])
        return logits[:, -1].argmax(dim=-1).cpu().tolist()
