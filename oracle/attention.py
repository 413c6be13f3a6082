"""CPU restatement of nifre's cached causal attention (oracle; test infrastructure only).

Follows ``src/inference/attention.py`` of jyotilakra92/nifre:

* ``attend_row``        -- ``Attention._forward_with_cache_row`` (``attention.py:106-142``)
  past K/V cast to the query dtype (``:122-123``), concatenated in front of the
  new K/V (``:126-127``), ``scores = q @ k^T`` in the query dtype (``:133``), the
  causal mask ``key > past_len + query`` when more than one query is new
  (``:135-137``, ``_causal_mask`` ``:144-152``), ``softmax(scores / sqrt(D))``
  (``:139``) and ``@ v`` (``:141``).
* ``forward_with_cache`` -- ``Attention._forward_with_cache`` (``attention.py:77-104``)
  row loop over a left-padded ``(B, T, H*D)`` batch: a prefill row keeps its
  last ``input_lens[i]`` tokens (``:83-93``), rows of ``out`` that are padding
  stay zero (``:79``), and each row does get -> append -> attend.
* ``full_causal``        -- ``Attention._forward_full_causal`` (``attention.py:59-75``).

Grouped-query attention (``Hq = group * Hkv``) is not expressible in the
reference, whose cache has a single head count.  The restatement stores the
``Hkv`` KV heads and expands them with ``repeat_interleave(group, dim=heads)``
right before the reference math, which is exactly the reference run on a cache
whose K/V heads were repeated (query head ``j`` reads KV head ``j // group``).
"""

from __future__ import annotations

import torch


def attend_row(q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
               past_k: torch.Tensor, past_v: torch.Tensor, group: int = 1) -> torch.Tensor:
    """One sequence's cached attention.

    q: (T, Hq, D); k_new, v_new: (T, Hkv, D) in q's dtype;
    past_k, past_v: (P, Hkv, D) in the cache dtype.  Returns (T, Hq, D).
    """
    T, Hq, D = q.shape
    queries = q.transpose(0, 1).unsqueeze(0)
    new_k = k_new.transpose(0, 1).unsqueeze(0)
    new_v = v_new.transpose(0, 1).unsqueeze(0)
    P = past_k.shape[0]
    if P > 0:
        pk = past_k.to(dtype=q.dtype).transpose(0, 1).unsqueeze(0)
        pv = past_v.to(dtype=q.dtype).transpose(0, 1).unsqueeze(0)
        keys = torch.cat([pk, new_k], dim=2)
        values = torch.cat([pv, new_v], dim=2)
    else:
        keys, values = new_k, new_v
    if group > 1:
        keys = keys.repeat_interleave(group, dim=1)
        values = values.repeat_interleave(group, dim=1)
    total = keys.shape[2]
    scores = queries @ keys.transpose(2, 3)
    if T > 1:
        key_idx = torch.arange(total)
        q_abs = torch.arange(T) + P
        scores.masked_fill_(key_idx.unsqueeze(0) > q_abs.unsqueeze(1), -torch.inf)
    w = torch.softmax(scores / D ** 0.5, dim=-1)
    ctx = w @ values
    return ctx.squeeze(0).transpose(0, 1).contiguous()


def forward_with_cache(store, layer: int, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                       num_q_heads: int, input_lens=None, slots=None) -> torch.Tensor:
    """Row loop of ``attention.py:77-104`` over an ``oracle.paged.OracleStore``.

    q: (B, T, Hq*D); k, v: (B, T, Hkv*D).  Returns (B, T, Hq*D) with padding rows zero.
    """
    B, T, _ = q.shape
    Hkv, D = store.H, store.D
    group = num_q_heads // Hkv
    out = torch.zeros_like(q)
    for i in range(B):
        slot = slots[i] if slots is not None else i
        n = int(input_lens[i]) if (input_lens is not None and T > 1) else T
        qi = q[i, T - n:].reshape(n, num_q_heads, D)
        ki = k[i, T - n:].reshape(n, Hkv, D)
        vi = v[i, T - n:].reshape(n, Hkv, D)
        past_k, past_v = store.get(slot, layer)
        store.append(slot, layer, ki.contiguous(), vi.contiguous())
        out[i, T - n:] = attend_row(qi, ki, vi, past_k, past_v, group).reshape(n, num_q_heads * D)
    return out


def ragged_layer(store, layer: int, seqs, group: int) -> list[torch.Tensor]:
    """Ragged form: ``seqs`` is a list of ``(slot, q (n,Hq,D), k (n,Hkv,D), v (n,Hkv,D))``.

    Rows are processed in list order, as the reference processes batch rows.
    Returns the per-sequence outputs (n, Hq, D).
    """
    outs = []
    for slot, qi, ki, vi in seqs:
        past_k, past_v = store.get(slot, layer)
        store.append(slot, layer, ki, vi)
        outs.append(attend_row(qi, ki, vi, past_k, past_v, group))
    return outs


def full_causal(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, num_heads: int) -> torch.Tensor:
    """``attention.py:59-75``: no cache, full causal attention over (B, T, H*D)."""
    B, T, HD = q.shape
    D = HD // num_heads
    qs = q.view(B, T, num_heads, D).transpose(1, 2)
    ks = k.view(B, T, num_heads, D).transpose(1, 2)
    vs = v.view(B, T, num_heads, D).transpose(1, 2)
    s = qs @ ks.transpose(2, 3)
    s.masked_fill_(torch.triu(torch.ones(T, T, dtype=torch.bool), diagonal=1), -torch.inf)
    w = torch.softmax(s / D ** 0.5, dim=-1)
    return (w @ vs).transpose(1, 2).contiguous().view(B, T, HD)


def attend_paged_fp32(q: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor,
                      blocks: list[int], ctx_len: int, group: int, causal_base: int | None = None):
    """Float32 attention of ``q`` (n, Hq, D) over the first ``ctx_len`` tokens of a paged sequence.

    Same math as ``attend_row`` once the new tokens are in the pool (the
    reference attends over ``past ++ new`` and the new rows are exactly what the
    append wrote); computed in float32 as a tolerance reference for 16-bit
    kernels.  ``causal_base`` is the absolute position of ``q[0]`` (masking
    ``key > causal_base + i``); None means ``ctx_len - n``.
    """
    n, Hq, D = q.shape
    bs = k_pool.shape[1]
    nb = (ctx_len + bs - 1) // bs
    idx = torch.tensor(blocks[:nb], dtype=torch.long)
    K = k_pool[idx].reshape(nb * bs, *k_pool.shape[2:])[:ctx_len].float()
    V = v_pool[idx].reshape(nb * bs, *v_pool.shape[2:])[:ctx_len].float()
    K = K.repeat_interleave(group, dim=1).transpose(0, 1)
    V = V.repeat_interleave(group, dim=1).transpose(0, 1)
    qs = q.float().transpose(0, 1)
    s = (qs @ K.transpose(1, 2)) / D ** 0.5
    base = ctx_len - n if causal_base is None else causal_base
    if n > 1 or causal_base is not None:
        key_idx = torch.arange(ctx_len)
        q_abs = torch.arange(n) + base
        s.masked_fill_(key_idx.unsqueeze(0) > q_abs.unsqueeze(1), -torch.inf)
    w = torch.softmax(s, dim=-1)
    return (w @ V).transpose(0, 1)
