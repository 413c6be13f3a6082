"""Model-agnostic attention over the B200 paged KV cache (drop-in for nifre's Attention).

Same constructor and ``forward(q, k, v, kv_cache=None, layer_id=None,
input_lens=None, cache_batch_indices=None)`` contract as jyotilakra92/nifre
``src/inference/attention.py:16-152``:

* ``q``/``k``/``v`` are projected ``(batch, seq, heads * head_dim)`` tensors;
  ``k``/``v`` may carry fewer (KV) heads than ``q`` (grouped-query attention,
  query head ``j`` reads KV head ``j // (Hq / Hkv)``);
* with a cache, each row appends its new K/V and attends causally over
  ``past + new`` with the query at absolute position ``past_len + i``
  (``attention.py:77-152``); a left-padded prefill row uses its last
  ``input_lens[i]`` tokens and its padding rows of the output stay zero
  (``:79-93``); ``pos`` advances after the last layer;
* without a cache it is full causal attention (``:59-75``);
* a missing ``layer_id`` with a cache raises ValueError (``:45-46``).

All rows of a call go through one ``nf_kv_append`` and one
``nf_paged_attention`` launch; the batch metadata is packed once per forward
(first layer) and reused by the other layers.  ``input_lens`` given as a CUDA
tensor costs one device->host read per forward (the reference reads it with
``.item()`` per row); pass a list or CPU tensor to avoid it.
"""

from __future__ import annotations

import math

import numpy as np
import torch
from torch import nn

from nifre_b200 import _lib
from nifre_b200.paged_kv_cache import PagedKVCache


class Attention(nn.Module):
    def __init__(self, num_heads, head_dim, layer_id=None, dropout=0.0):
        super().__init__()
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.d_out = num_heads * head_dim
        self.layer_id = layer_id
        self.dropout = nn.Dropout(dropout)

    def forward(self, q, k, v, kv_cache=None, layer_id=None, input_lens=None, cache_batch_indices=None):
        lid = layer_id if layer_id is not None else self.layer_id
        if kv_cache is None:
            return self._forward_full_causal(q, k, v)
        if lid is None:
            raise ValueError("layer_id is required when kv_cache is set")
        if not isinstance(kv_cache, PagedKVCache):
            raise TypeError("nifre_b200.Attention runs on nifre_b200.PagedKVCache or nifre_b200.KVCache")
        return self._forward_with_cache(q, k, v, kv_cache, lid, input_lens, cache_batch_indices)

    # ------------------------------------------------------------------ cached path
    def _forward_with_cache(self, q, k, v, cache: PagedKVCache, layer_id, input_lens, cache_batch_indices):
        # The reference attends in q's dtype with the step's new K/V at projection precision and the cached
        # ones cast to q's dtype (attention.py:121-133); torch's matmul there needs q, k and v of one dtype.
        # This path attends in the cache dtype, which is the same computation exactly when q/k/v share the
        # cache's dtype (as every reference caller has it: engine.py:218-227 passes the model dtype); other
        # combinations are refused before any launch rather than computed differently.
        if not (q.dtype == k.dtype == v.dtype == cache.dtype):
            raise ValueError(f"q/k/v dtypes ({q.dtype}, {k.dtype}, {v.dtype}) must equal the cache dtype "
                             f"{cache.dtype}: create the cache with the model's dtype")
        B, T, _ = q.shape
        if cache_batch_indices is None:
            slots = tuple(range(B))
        elif torch.is_tensor(cache_batch_indices):
            slots = tuple(cache_batch_indices.tolist())
        else:
            slots = tuple(cache_batch_indices)  # compared as given; made ints below when a plan is built
        if input_lens is not None and T > 1:
            lens = input_lens.tolist() if torch.is_tensor(input_lens) else [int(x) for x in input_lens]
            lens_key = tuple(lens)
            padded = any(n != T for n in lens)
        else:  # every row has T new tokens
            lens, lens_key, padded = None, None, False
        key = (slots, lens_key, T, B)
        plan = cache._plan
        if plan is None or plan.key != key or plan.closed:
            slots = [int(s) for s in slots]
            if lens is None:
                lens = [T] * B
            starts = [i * T + (T - n) for i, n in enumerate(lens)]
            plan = cache.plan(slots, lens, starts, q_heads=self.num_heads)
            plan.key = key
        q2 = q.reshape(B * T, q.shape[-1])
        k2 = k.reshape(B * T, k.shape[-1])
        v2 = v.reshape(B * T, v.shape[-1])
        if k2.stride(1) != 1:
            k2 = k2.contiguous()
        if v2.stride(1) != 1:
            v2 = v2.contiguous()
        qk = q2 if q2.stride(1) == 1 else q2.contiguous()
        # padding rows of a left-padded prefill stay zero (attention.py:79); without padding every row is written
        ex = cache.exchange
        if ex is not None:
            # KV heads sharded over the ranks of a PeerExchange: the kernels write this rank's heads into every
            # rank's gathered buffer; the result is the gathered output of all heads
            if padded:
                raise ValueError("a sharded cache (exchange set) takes unpadded rows only")
            slot = ex.slot_for(layer_id, cache.steps_closed, cache.num_layers)
            cache.append_step(layer_id, k2, v2, plan)
            cache.attention_step(layer_id, qk, plan, ex.out(slot, B * T), scale=1.0 / math.sqrt(self.head_dim),
                                 exchange=ex)
            return ex.gathered(slot, B * T).view(B, T, -1)
        out = (torch.zeros if padded else torch.empty)((B * T, q.shape[-1]), dtype=cache.dtype, device=q.device)
        cache.append_step(layer_id, k2, v2, plan)
        cache.attention_step(layer_id, qk, plan, out, scale=1.0 / math.sqrt(self.head_dim))
        return out.view(B, T, -1)

    # ------------------------------------------------------------------ no-cache path
    def _forward_full_causal(self, q, k, v):
        """Full causal attention through the same kernels: each row's K/V is a one-block pool."""
        return causal_attention(q, k, v, self.head_dim)


def causal_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, head_dim: int) -> torch.Tensor:
    """Causal attention over (B, T, H*D) tensors without a cache (attention.py:59-75).

    Row b of ``k``/``v`` is used in place as block b of a pool whose block
    size is T, with the identity block table.  16-bit tensors with head_dim
    64 or 128 (and 1, 2, 4 or 8 query heads per KV head) go to the
    tensor-core prefill kernel, every row one chunk at position 0; other
    shapes to the split-K kernel, every query i of row b a work item over
    keys [0, i].
    """
    _lib.require_cuda(q, "q")
    B, T, hqd = q.shape
    dtype = q.dtype
    k = k.to(dtype).contiguous()
    v = v.to(dtype).contiguous()
    q = q.contiguous()
    hkv = k.shape[-1] // head_dim
    hq = hqd // head_dim
    if (dtype in (torch.bfloat16, torch.float16) and head_dim in (64, 128) and hkv > 0 and hq % hkv == 0
            and hq // hkv in (1, 2, 4, 8)):
        return _causal_tensor_core(q, k, v, head_dim, hq, hkv)
    dev = q.device
    n_tok = B * T
    split = 128 * max(1, math.ceil(T / 128))
    max_units = n_tok  # one unit per query: kv_len <= T <= split
    seqs = np.stack([np.arange(B), np.arange(B) * T, np.full(B, T), np.zeros(B)], 1).astype(np.int32)
    seqs_d = torch.from_numpy(seqs.reshape(-1)).to(dev)
    bt = torch.arange(B, dtype=torch.int32, device=dev).view(B, 1)
    slot_mapping = torch.empty(n_tok, dtype=torch.int32, device=dev)
    src_rows = torch.empty_like(slot_mapping)
    items = torch.empty(4 * n_tok, dtype=torch.int32, device=dev)
    units = torch.empty(_lib.UNIT_FIELDS * max_units, dtype=torch.int32, device=dev)
    counts = torch.empty(4, dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = _lib.stream_handle(dev)
    lib = _lib.load()
    _lib.check(lib.nf_pack_step(seqs_d.data_ptr(), B, None, 0, bt.data_ptr(), B, 1, T, B, split, None, None,
                                slot_mapping.data_ptr(), src_rows.data_ptr(), None, items.data_ptr(),
                                units.data_ptr(), counts.data_ptr(), n_tok, max_units, status.data_ptr(),
                                stream), "nf_pack_step")
    pf, ci = _lib.workspace_sizes(max_units, n_tok, hq, hkv, head_dim, dtype)
    ws = torch.empty(max(pf, 1), dtype=torch.float32, device=dev)
    cnt = torch.zeros(max(ci, 1), dtype=torch.int32, device=dev)
    out = torch.empty_like(q)
    _lib.check(lib.nf_paged_attention(
        out.data_ptr(), hqd, q.data_ptr(), hqd, k.data_ptr(), v.data_ptr(), _lib.dtype_code(dtype),
        hq, hkv, head_dim, T, B, bt.data_ptr(), 1, items.data_ptr(), units.data_ptr(), counts.data_ptr(),
        n_tok, max_units, split, 1.0 / math.sqrt(head_dim), ws.data_ptr(), ws.numel(), cnt.data_ptr(),
        cnt.numel(), status.data_ptr(), stream), "nf_paged_attention")
    return out


def _causal_tensor_core(q, k, v, head_dim, hq, hkv):
    """The no-cache path on nf_prefill_attention: row b of k/v is block b of a pool whose block size is T
    rounded up to 16 (zero-padded when T is not a multiple of 16; the padding keys lie past every query's
    causal limit), and the row's queries are chunks at position 0."""
    from nifre_b200.paged_kv_cache import _prefill_order

    B, T, hqd = q.shape
    dev = q.device
    bs = (T + 15) // 16 * 16
    if bs != T:
        kp = torch.zeros(B, bs, hkv * head_dim, dtype=q.dtype, device=dev)
        vp = torch.zeros_like(kp)
        kp[:, :T] = k
        vp[:, :T] = v
    else:
        kp, vp = k, v
    lib = _lib.load()
    tt = lib.nf_prefill_tile_rows(head_dim) // (hq // hkv)  # tokens per work item
    t0 = np.arange(0, T, tt, dtype=np.int64)
    b = np.repeat(np.arange(B, dtype=np.int64), len(t0))
    t0 = np.tile(t0, B)
    tiles = np.stack([b, b * T + t0, np.minimum(tt, T - t0), t0], axis=1)
    order = _prefill_order([tuple(r) for r in tiles.tolist()], hkv)
    meta = torch.from_numpy(np.concatenate([tiles.reshape(-1), order]).astype(np.int32)).to(dev)
    bt = torch.arange(B, dtype=torch.int32, device=dev).view(B, 1)
    queue = torch.zeros(2, dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    out = torch.empty_like(q)
    n_tiles = len(tiles)
    _lib.check(lib.nf_prefill_attention(
        out.data_ptr(), hqd, q.data_ptr(), hqd, B * T, kp.data_ptr(), vp.data_ptr(), _lib.dtype_code(q.dtype),
        hq, hkv, head_dim, bs, B, bt.data_ptr(), 1, meta.data_ptr(), n_tiles, meta.data_ptr() + 16 * n_tiles,
        queue.data_ptr(), 1.0 / math.sqrt(head_dim), status.data_ptr(), _lib.stream_handle(dev)),
        "nf_prefill_attention")
    return out
