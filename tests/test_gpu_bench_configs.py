"""Parity on the benchmark configurations themselves (B200).

* The Llama-3-8B-shaped long-context decode: head_dim 128, 32 query heads
  over 8 KV heads, contexts drawn from U[4096, 32768] with the benchmark's
  seed (a subset that includes the longest context), split-K units sized as
  for the whole 256-sequence batch and as for the subset alone.
* The mixed continuous-batching step on the Llama-3.2-1B shape exactly as
  the benchmark builds it: 4 prefill chunks of 512 tokens continuing cached
  prefixes U[0, 2048] plus 96 decodes over contexts U[256, 2048], one plan,
  chunks on the tensor-core prefill kernel and decodes on the split-K kernel.

Outputs are bfloat16 within rtol/atol 2e-2 of the float32 oracle
(``oracle.attention.attend_paged_fp32``: the reference's per-row cached
attention, attention.py:106-152, with grouped-query heads expanded).  Each
sequence's blocks are gathered on the device before the oracle runs, so the
multi-GB pools never travel to the host whole.
"""

import numpy as np
import pytest
import torch

from oracle.attention import attend_paged_fp32

pytestmark = pytest.mark.gpu

DEV = "cuda"
TOL = dict(rtol=2e-2, atol=2e-2)


def _fill(cache, slots, lens, g, layers=1, group_tokens=1 << 19):
    """Append N(0, 1) keys and values for `lens[i]` tokens of `slots[i]`, in groups of sequences."""
    groups, cur = [], []
    for i in range(len(slots)):
        if cur and sum(lens[j] for j in cur) + lens[i] > group_tokens:
            groups.append(cur)
            cur = []
        cur.append(i)
    groups.append(cur)
    H = cache.n_heads * cache.head_dim
    for grp in groups:
        n = [lens[i] for i in grp]
        plan = cache.plan([slots[i] for i in grp], n, np.cumsum([0] + n[:-1]).tolist())
        k = torch.empty(sum(n), H, device=DEV, dtype=cache.dtype)
        v = torch.empty_like(k)
        for layer in range(layers):
            k.normal_(generator=g)
            v.normal_(generator=g)
            cache.append_step(layer, k, v, plan)


def _oracle(cache, slot, q_rows, kv_len, group, causal_base=None):
    """The oracle over one sequence, its blocks gathered on the device first."""
    bs = cache.block_size
    nb = (kv_len + bs - 1) // bs
    idx = torch.tensor(cache.block_tables[slot].physical_blocks()[:nb], device=DEV)
    kp = cache.k[0].index_select(0, idx).cpu()
    vp = cache.v[0].index_select(0, idx).cpu()
    return attend_paged_fp32(q_rows, kp, vp, list(range(nb)), kv_len, group, causal_base=causal_base)


@pytest.mark.parametrize("unit_sizing", ["whole batch", "subset"])
def test_long_context_decode_8b_shape(unit_sizing):
    from nifre_b200 import PagedKVCache
    Hq, Hkv, D, bs = 32, 8, 128, 16
    population = np.random.default_rng(0).integers(4096, 32768 + 1, size=256)  # the benchmark's contexts
    pick = sorted({int(np.argmax(population)), int(np.argmin(population))}
                  | set(np.random.default_rng(7).choice(256, size=8, replace=False).tolist()))
    ctx = [int(population[i]) for i in pick]
    assert max(ctx) > 32000
    B = len(ctx)
    cache = PagedKVCache(1, max(ctx) + 8, Hkv, D, device=DEV, dtype=torch.bfloat16, block_size=bs,
                         enable_prefix_cache=False, num_blocks=sum((c + 8 + bs - 1) // bs for c in ctx))
    cache.init_batch(B)
    g = torch.Generator().manual_seed(5)
    cache.block_allocator.set_free_order(torch.randperm(cache.num_blocks, generator=g).tolist())
    gd = torch.Generator(device=DEV).manual_seed(5)
    _fill(cache, list(range(B)), ctx, gd)
    q = torch.randn(B, Hq * D, generator=g).to(torch.bfloat16).to(DEV)
    kn = torch.randn(B, Hkv * D, generator=g).to(torch.bfloat16).to(DEV)
    vn = torch.randn(B, Hkv * D, generator=g).to(torch.bfloat16).to(DEV)
    # split-K units as the 256-sequence batch gets them (each layer of that workload), or as for this batch
    split = cache.split_for(int(population.sum()) + 256) if unit_sizing == "whole batch" else None
    plan = cache.plan(list(range(B)), [1] * B, list(range(B)), split=split, q_heads=Hq)
    cache.append_step(0, kn, vn, plan)
    out = torch.zeros_like(q)
    cache.attention_step(0, q, plan, out)
    torch.cuda.synchronize()
    cache.check_status()
    if unit_sizing == "whole batch":
        assert plan.split >= 4096  # several thousand keys per unit, as in the benchmark
    assert plan.max_units > B  # every sequence is split into several parts
    for b in range(B):
        ref = _oracle(cache, b, q[b].view(1, Hq, D).cpu(), ctx[b] + 1, Hq // Hkv)
        torch.testing.assert_close(out[b].view(Hq, D).float().cpu(), ref[0], **TOL)


def test_mixed_step_1b_shape():
    from nifre_b200 import PagedKVCache
    Hq, Hkv, D, bs, C = 32, 8, 64, 16, 512
    rng = np.random.default_rng(0)  # the benchmark's mixed-step shape
    prefix = rng.integers(0, 2048 + 1, size=4).tolist()
    dctx = rng.integers(256, 2048 + 1, size=96).tolist()
    P, ND = len(prefix), len(dctx)
    B = P + ND
    ctx = prefix + dctx
    cache = PagedKVCache(1, max(max(prefix) + C, max(dctx) + 1) + 8, Hkv, D, device=DEV, dtype=torch.bfloat16,
                         block_size=bs, enable_prefix_cache=False)
    cache.init_batch(B)
    g = torch.Generator().manual_seed(0)
    cache.block_allocator.set_free_order(torch.randperm(cache.num_blocks, generator=g).tolist())
    gd = torch.Generator(device=DEV).manual_seed(0)
    fill = [i for i in range(B) if ctx[i] > 0]
    _fill(cache, fill, [ctx[i] for i in fill], gd)
    q_lens = [C] * P + [1] * ND
    starts = np.cumsum([0] + q_lens[:-1]).tolist()
    T = sum(q_lens)
    q = torch.randn(T, Hq * D, device=DEV, dtype=torch.bfloat16, generator=gd)
    k = torch.randn(T, Hkv * D, device=DEV, dtype=torch.bfloat16, generator=gd)
    v = torch.randn(T, Hkv * D, device=DEV, dtype=torch.bfloat16, generator=gd)
    plan = cache.plan(list(range(B)), q_lens, starts, q_heads=Hq)
    from nifre_b200 import _lib
    tokens_per_tile = _lib.load().nf_prefill_tile_rows(D) // (Hq // Hkv)
    assert plan.n_tiles == P * C // tokens_per_tile  # every chunk on the tensor-core kernel
    assert plan.decode_units >= ND
    cache.append_step(0, k, v, plan)
    out = torch.full_like(q, float("nan"))
    cache.attention_step(0, q, plan, out)
    torch.cuda.synchronize()
    cache.check_status()
    assert torch.isfinite(out).all()
    for s in range(B):
        n, st = q_lens[s], starts[s]
        ref = _oracle(cache, s, q[st:st + n].view(n, Hq, D).cpu(), ctx[s] + n, Hq // Hkv, causal_base=ctx[s])
        torch.testing.assert_close(out[st:st + n].view(n, Hq, D).float().cpu(), ref, **TOL)
