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
"""

from __future__ import annotations

from typing import List, Optional

import numpy as np
import torch

from .batching import batch_token_ids
from .data_model import InferenceRequest


class ModelRunner:
    def __init__(self, model, device):
        self.model = model
        self.device = torch.device(device)
        self.model.eval()

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
        plan = cache.plan(slots, lens, starts.tolist(), q_heads=getattr(self.model.config, "n_heads", None))
        dev = self.device
        host = torch.from_numpy(np.concatenate([np.asarray(ids, np.int64), positions.astype(np.int64),
                                                np.asarray(sample, np.int64)])).pin_memory()
        buf = host.to(dev, non_blocking=True)
        T, S = len(ids), len(sample)
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
