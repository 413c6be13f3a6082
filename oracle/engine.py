"""CPU restatement of the reference's greedy generation with a KV cache (oracle; test infrastructure only).

Used as the CPU baseline and the reference arm of the end-to-end engine
workload in ``bench.py``: one request at a time, every layer of every step
running the reference's per-row cached attention (``attend_row``:
``src/inference/attention.py:106-142`` of jyotilakra92/nifre) over a per-row
past that grows by concatenation (``PagedKVCache.get`` + ``append``,
``paged_kv_cache.py:107-142``: the reference gathers and re-concatenates
the whole past every layer and step).  The rest of the forward is the
reference GPT (``src/inference/models/gpt.py:103-141``): token + position
embeddings, per block ``x + out_proj(attn(norm1(x)))`` then
``x + ff(norm2(x))``, final norm, output head, greedy ``argmax``
(``src/sampler.py:4-6``) on the last position.  The modules themselves are
the ones of the model passed in (a CPU copy), so the arithmetic outside the
attention is the module code both sides share.
"""

from __future__ import annotations

import time

import torch

from .attention import attend_row


@torch.no_grad()
def _forward(model, ids: list[int], pos0: int, past: list) -> torch.Tensor:
    """Logits of the last of ``ids`` (tokens at positions pos0 ..), appending their K/V to ``past``."""
    T = len(ids)
    x = model.token_embedding(torch.tensor(ids)) + model.position_embedding(torch.arange(pos0, pos0 + T))
    for layer, block in enumerate(model.trf_blocks):
        att = block.att
        H, D = att.num_heads, att.head_dim
        h = block.norm1(x)
        q = att.W_query(h).view(T, H, D)
        k = att.W_key(h).view(T, H, D)
        v = att.W_value(h).view(T, H, D)
        pk, pv = past[layer]
        ctx = attend_row(q, k, v, pk, pv)  # reference per-row attention over past ++ new
        past[layer] = (torch.cat([pk, k]), torch.cat([pv, v]))
        x = x + att.out_proj(ctx.reshape(T, H * D))
        x = x + block.ff(block.norm2(x))
    return model.out_head(model.final_norm(x[-1:]))[0]


@torch.no_grad()
def greedy_generate(model, prompt: list[int], new_tokens: int) -> tuple[list[int], float, int]:
    """Greedy continuation of one prompt on the CPU.

    Returns the new tokens, the seconds spent in decode steps (after the
    prompt's prefill) and the number of decode steps timed.
    """
    blocks = model.trf_blocks
    H, D = blocks[0].att.num_heads, blocks[0].att.head_dim
    past = [(torch.empty(0, H, D), torch.empty(0, H, D)) for _ in blocks]
    logits = _forward(model, prompt, 0, past)
    out = [int(torch.argmax(logits))]
    t0 = time.perf_counter()
    for i in range(new_tokens - 1):
        logits = _forward(model, [out[-1]], len(prompt) + i, past)
        out.append(int(torch.argmax(logits)))
    return out, time.perf_counter() - t0, new_tokens - 1
