"""CUDA path vs the reference outputs and the CPU oracle (needs a B200).

Tolerances: float32 pools within rtol 1e-4 / atol 1e-5 of the reference's
float32 math; bfloat16 within rtol 2e-2 / atol 2e-2 (the stated tolerance of
the attention outputs).  Pool contents, block tables and pos are bit-exact.
"""

import math

import pytest
import torch

from oracle.attention import attend_paged_fp32, full_causal
from oracle.paged import OracleStore

pytestmark = pytest.mark.gpu

DEV = "cuda"
RAGGED = ("mha_fp32", "gqa_bf16", "gqa_fp32", "gqa_d128_bf16")


def _tol(dtype):
    return dict(rtol=1e-4, atol=1e-5) if dtype == torch.float32 else dict(rtol=2e-2, atol=2e-2)


def _dtype(name):
    return {"torch.float32": torch.float32, "torch.bfloat16": torch.bfloat16, "torch.float16": torch.float16}[name]


@pytest.fixture(scope="module", autouse=True)
def _lib_built():
    from nifre_b200 import _lib
    _lib.load()


def _written(tables, pos, bs):
    b, o = [], []
    for slot, blocks in enumerate(tables):
        for t in range(int(pos[slot])):
            b.append(blocks[t // bs])
            o.append(t % bs)
    return torch.tensor(b), torch.tensor(o)


@pytest.mark.parametrize("name", RAGGED)
def test_golden_ragged_replay(golden_paged, name):
    from nifre_b200 import Attention, PagedKVCache
    case = golden_paged[name]
    dt = _dtype(case["dtype"])
    B = len(case["prompt_lens"])
    cache = PagedKVCache(case["L"], case["max_seq_len"], case["Hkv"], case["D"], device=DEV, dtype=dt,
                         block_size=case["bs"], enable_prefix_cache=False)
    cache.init_batch(B)
    assert cache.num_blocks == case["num_blocks"]
    if case["free_order"] is not None:
        cache.block_allocator.set_free_order(case["free_order"])
    attn = Attention(case["Hq"], case["D"])
    for step in case["steps"]:
        il = torch.tensor(step["lens"]) if step["kind"] == "prefill" else None
        for layer in range(case["L"]):
            out = attn(step["q"].to(DEV), step["k"].to(DEV), step["v"].to(DEV), kv_cache=cache,
                       layer_id=layer, input_lens=il, cache_batch_indices=step["slots"])
            torch.testing.assert_close(out.cpu().float(), step["outs"][layer].float(), **_tol(dt))
            if step["kind"] == "prefill":  # padding rows stay exactly zero
                for r, n in enumerate(step["lens"]):
                    assert torch.count_nonzero(out[r, : out.shape[1] - n]) == 0
        assert [t.physical_blocks() for t in cache.block_tables] == step["tables"]
        assert cache.pos.cpu().tolist() == step["pos"].tolist()
        for s in range(B):
            assert cache.device_block_table(s) == step["tables"][s]
    b, o = _written(case["steps"][-1]["tables"], case["steps"][-1]["pos"], case["bs"])
    k_all = torch.stack([t.cpu() for t in cache.k])
    v_all = torch.stack([t.cpu() for t in cache.v])
    assert torch.equal(k_all[:, b, o], case["k_pool"][:, b, o])
    assert torch.equal(v_all[:, b, o], case["v_pool"][:, b, o])
    cache.check_status()


def test_golden_smoke_sequence(golden_paged):
    """The reference attention smoke sequence on the paged cache (bs 8, fp32, head_dim 4)."""
    from nifre_b200 import Attention, PagedKVCache
    case = golden_paged["smoke_paged"]
    H, D, L = case["H"], case["D"], case["L"]
    attn = Attention(H, D)
    cache = PagedKVCache(L, case["max_seq_len"], H, D, device=DEV, dtype=torch.float32, block_size=case["bs"])
    cache.init_batch(1)
    for i, call in enumerate(case["calls"]):
        if i == 2:
            cache.free()
            cache.init_batch(2)
        before = [cache.length(s) for s in range(cache.batch_size)]
        for layer in range(L):
            out = attn(call["q"].to(DEV), call["k"].to(DEV), call["v"].to(DEV), kv_cache=cache, layer_id=layer,
                       input_lens=call["input_lens"], cache_batch_indices=call["slots"])
            torch.testing.assert_close(out.cpu(), call["outs"][layer], rtol=1e-4, atol=1e-5)
            if layer < L - 1:  # pos advances only after the last layer
                assert [cache.length(s) for s in range(cache.batch_size)] == before
        assert cache.pos.cpu().tolist() == call["pos"].tolist()
        assert [t.physical_blocks() for t in cache.block_tables] == call["tables"]
    cache.check_status()


def _random_cache(Hq, Hkv, D, bs, ctx_lens, dtype, seed, L=1, shuffle=True, room=8):
    """Fill a cache with N(0,1) keys for the given contexts through the prefill path
    (``room`` more tokens fit after the longest context)."""
    from nifre_b200 import PagedKVCache
    g = torch.Generator().manual_seed(seed)
    B = len(ctx_lens)
    max_len = max(ctx_lens) + room
    cache = PagedKVCache(L, max_len, Hkv, D, device=DEV, dtype=dtype, block_size=bs, enable_prefix_cache=False)
    cache.init_batch(B)
    if shuffle:
        cache.block_allocator.set_free_order(torch.randperm(cache.num_blocks, generator=g).tolist())
    T = sum(ctx_lens)
    k = torch.randn(T, Hkv * D, generator=g).to(dtype).to(DEV)
    v = torch.randn(T, Hkv * D, generator=g).to(dtype).to(DEV)
    starts = [sum(ctx_lens[:i]) for i in range(B)]
    plan = cache.plan(list(range(B)), ctx_lens, starts)
    for layer in range(L):
        cache.append_step(layer, k, v, plan)
    return cache, g


@pytest.mark.parametrize("split", [None, 128])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("D,Hq,Hkv", [(64, 32, 8), (128, 32, 8), (64, 12, 12), (128, 8, 1), (128, 16, 2), (64, 4, 1), (64, 8, 2)])
def test_decode_vs_oracle(dtype, D, Hq, Hkv, split):
    ctx = [1, 15, 16, 17, 100, 513, 1000, 2049]
    cache, g = _random_cache(Hq, Hkv, D, 16, ctx, dtype, seed=D + Hq)
    B = len(ctx)
    q = torch.randn(B, Hq * D, generator=g).to(dtype).to(DEV)
    kn = torch.randn(B, Hkv * D, generator=g).to(dtype).to(DEV)
    vn = torch.randn(B, Hkv * D, generator=g).to(dtype).to(DEV)
    plan = cache.plan(list(range(B)), [1] * B, list(range(B)), split=split)
    cache.append_step(0, kn, vn, plan)
    out = torch.zeros_like(q)
    cache.attention_step(0, q, plan, out)
    # the plan closed on the last layer: pos advanced by one
    assert cache.pos.cpu().tolist() == [c + 1 for c in ctx]
    for b in range(B):
        ref = attend_paged_fp32(q[b].view(1, Hq, D).cpu(), cache.k[0].cpu(), cache.v[0].cpu(),
                                cache.block_tables[b].physical_blocks(), ctx[b] + 1, Hq // Hkv)
        torch.testing.assert_close(out[b].view(Hq, D).float().cpu(), ref[0], **_tol(dtype))
    cache.check_status()


def test_pack_first_item_with_units_and_mixed_merge():
    """counts[2] carries, from bit 2, the first item with split-K units: a mixed step's prefill rows (listed
    first, served by the prefill kernel) have none, so the decode launch's end-of-launch merge starts after
    them.  The step's decode rows (several parts each) still match the oracle."""
    import numpy as np
    from oracle.attention import attend_paged_fp32
    ctx = [300, 0, 700, 900, 1500]
    cache, g = _random_cache(32, 8, 64, 16, [c if c else 16 for c in ctx], torch.bfloat16, seed=21, room=64)
    q_lens = [40, 24, 1, 1, 1]  # two prefill rows (>= 16 new tokens), then three decodes
    B, T = len(q_lens), sum(q_lens)
    before = [cache.length(s) for s in range(B)]
    starts = np.cumsum([0] + q_lens[:-1]).tolist()
    plan = cache.plan(list(range(B)), q_lens, starts, q_heads=32, split=128)
    assert plan.n_tiles > 0
    flags = int(plan.counts[2].item())
    assert flags >> 2 == 64 and flags & 2  # items 0..63 are the prefill rows'; the decodes have several units
    q = torch.randn(T, 32 * 64, generator=g).to(torch.bfloat16).to(DEV)
    k = torch.randn(T, 8 * 64, generator=g).to(torch.bfloat16).to(DEV)
    cache.append_step(0, k, k, plan)
    out = torch.zeros_like(q)
    cache.attention_step(0, q, plan, out)
    cache.check_status()
    kp, vp = cache.k[0].cpu(), cache.v[0].cpu()
    for b in (2, 3, 4):
        ref = attend_paged_fp32(q[starts[b]].view(1, 32, 64).cpu(), kp, vp, cache.block_tables[b].physical_blocks(),
                                before[b] + 1, 4)
        torch.testing.assert_close(out[starts[b]].view(32, 64).float().cpu(), ref[0], rtol=2e-2, atol=2e-2)


def test_pack_unit_list():
    """Every key range of every item appears once with its part index; the last field holds the item's
    part count (low 16 bits) and unit count (high bits; the same here: no cascade parts); the units of
    sequences at the step's split come first, then the short-unit tail, each in item order."""
    import numpy as np
    rng = np.random.default_rng(3)
    ctx = rng.integers(1, 3000, size=64).tolist()
    cache, _ = _random_cache(32, 8, 64, 16, ctx, torch.bfloat16, seed=3)  # a full KV-head group per CTA
    B, split = len(ctx), 128
    plan = cache.plan(list(range(B)), [1] * B, list(range(B)), split=split)
    kv = np.array(ctx) + 1
    us = plan.seq_split.astype(np.int64)
    assert (us < split).any() and (us == split).any()
    nsp = (kv + us - 1) // us
    n_units = int(nsp.sum())
    counts = plan.counts.cpu().numpy()
    assert counts[0] == B and counts[1] == n_units == plan.max_units
    items = plan.items.cpu().numpy().reshape(-1, 4)[:B]
    units = plan.units.cpu().numpy().reshape(-1, 8)[:n_units]
    assert (items[:, 2] == kv).all()
    assert (items[:, 3] == np.concatenate([[0], np.cumsum(nsp)[:-1]])).all()  # unit_base
    seen = set()
    for t, slot, q_row, part, k0, k1, ub, n in units.tolist():
        assert (slot, q_row, ub, n & 0xFFFF, n >> 16) == (t, t, items[t, 3], nsp[t], nsp[t])
        assert k0 == part * us[t] and k1 == min(k0 + us[t], kv[t])
        seen.add((t, part))
    assert seen == {(t, j) for t in range(B) for j in range(nsp[t])}
    fine = us[units[:, 0]] < split
    n_bulk = int(nsp[us == split].sum())
    assert not fine[:n_bulk].any() and fine[n_bulk:].all()
    key = units[:, 0].astype(np.int64) * 100000 + units[:, 3]  # (item, part)
    assert (np.diff(key[:n_bulk]) > 0).all() and (np.diff(key[n_bulk:]) > 0).all()
    cache.check_status()


@pytest.mark.parametrize("D,Hq,Hkv", [(64, 32, 8), (128, 32, 8)])
def test_decode_many_seqs_vs_oracle(D, Hq, Hkv):
    """A decode batch of 64 ragged contexts with a small split: many parts, merges and queue rounds."""
    import numpy as np
    dtype = torch.bfloat16
    ctx = np.random.default_rng(D).integers(1, 2500, size=64).tolist()
    cache, g = _random_cache(Hq, Hkv, D, 16, ctx, dtype, seed=11)
    B = len(ctx)
    q = torch.randn(B, Hq * D, generator=g).to(dtype).to(DEV)
    kn = torch.randn(B, Hkv * D, generator=g).to(dtype).to(DEV)
    vn = torch.randn(B, Hkv * D, generator=g).to(dtype).to(DEV)
    plan = cache.plan(list(range(B)), [1] * B, list(range(B)), split=128)
    cache.append_step(0, kn, vn, plan)
    out = torch.zeros_like(q)
    for _ in range(2):  # the second launch runs on the counters the first left behind
        out.zero_()
        cache.attention_step(0, q, plan, out)
    kp, vp = cache.k[0].cpu(), cache.v[0].cpu()
    for b in range(B):
        ref = attend_paged_fp32(q[b].view(1, Hq, D).cpu(), kp, vp, cache.block_tables[b].physical_blocks(),
                                ctx[b] + 1, Hq // Hkv)
        torch.testing.assert_close(out[b].view(Hq, D).float().cpu(), ref[0], **_tol(dtype))
    cache.check_status()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_chunked_prefill_with_past_vs_oracle(dtype):
    """Prefill chunks continuing cached prefixes (mask key > past + i), mixed with decodes."""
    Hq, Hkv, D = 16, 4, 64
    past = [0, 5, 16, 300, 40]
    cache, g = _random_cache(Hq, Hkv, D, 16, [max(p, 1) for p in past], dtype, seed=7)
    # slot 0 starts empty: reset it
    cache.reset_slot(0)
    qlens = [37, 1, 64, 1, 130]
    T = sum(qlens)
    q = torch.randn(T, Hq * D, generator=g).to(dtype).to(DEV)
    k = torch.randn(T, Hkv * D, generator=g).to(dtype).to(DEV)
    v = torch.randn(T, Hkv * D, generator=g).to(dtype).to(DEV)
    starts = [sum(qlens[:i]) for i in range(len(qlens))]
    before = [cache.length(s) for s in range(len(qlens))]
    plan = cache.plan(list(range(len(qlens))), qlens, starts)
    cache.append_step(0, k, v, plan)
    out = torch.zeros_like(q)
    cache.attention_step(0, q, plan, out)
    for s, (st, n) in enumerate(zip(starts, qlens)):
        ref = attend_paged_fp32(q[st:st + n].view(n, Hq, D).cpu(), cache.k[0].cpu(), cache.v[0].cpu(),
                                cache.block_tables[s].physical_blocks(), before[s] + n, Hq // Hkv,
                                causal_base=before[s])
        torch.testing.assert_close(out[st:st + n].view(n, Hq, D).float().cpu(), ref, **_tol(dtype))
    cache.check_status()


def test_append_conversion_bit_exact():
    """float32 projections into a bf16 pool: rounding identical to torch's copy (paged_kv_cache.py:114-115)."""
    from nifre_b200 import PagedKVCache
    g = torch.Generator().manual_seed(3)
    cache = PagedKVCache(2, 64, 4, 64, device=DEV, dtype=torch.bfloat16, block_size=16)
    cache.init_batch(3)
    lens = [7, 33, 1]
    T = sum(lens)
    k = (torch.randn(T, 256, generator=g) * 3).to(DEV)
    v = (torch.randn(T, 256, generator=g) * 3).to(DEV)
    plan = cache.plan([0, 1, 2], lens, [0, 7, 40])
    for layer in range(2):
        cache.append_step(layer, k, v, plan)
    for s, (st, n) in enumerate(zip([0, 7, 40], lens)):
        kk, vv = cache.get(s, 1)
        assert torch.equal(kk.reshape(n, -1), k[st:st + n].to(torch.bfloat16))
        assert torch.equal(vv.reshape(n, -1), v[st:st + n].to(torch.bfloat16))
    cache.check_status()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_no_cache_causal_vs_oracle(dtype):
    from nifre_b200 import Attention
    g = torch.Generator().manual_seed(5)
    B, T, H, D = 3, 37, 4, 64
    q, k, v = (torch.randn(B, T, H * D, generator=g).to(dtype) for _ in range(3))
    out = Attention(H, D)(q.to(DEV), k.to(DEV), v.to(DEV))
    ref = full_causal(q.float(), k.float(), v.float(), H)
    torch.testing.assert_close(out.float().cpu(), ref, **_tol(dtype))


@pytest.mark.parametrize("B,T,H,D", [(2, 300, 8, 64), (3, 64, 4, 128), (1, 1000, 2, 64), (2, 17, 16, 64)])
def test_no_cache_causal_tensor_core_vs_oracle(B, T, H, D):
    """The no-cache path on the tensor-core prefill kernel (T a multiple of 16 or padded to one)."""
    from nifre_b200 import Attention
    g = torch.Generator().manual_seed(B * T + D)
    q, k, v = (torch.randn(B, T, H * D, generator=g).to(torch.bfloat16) for _ in range(3))
    out = Attention(H, D)(q.to(DEV), k.to(DEV), v.to(DEV))
    ref = full_causal(q.float(), k.float(), v.float(), H)
    torch.testing.assert_close(out.float().cpu(), ref, rtol=2e-2, atol=2e-2)


def test_errors_before_launch():
    from nifre_b200 import BlockPoolExhaustedError, PagedKVCache
    cache = PagedKVCache(1, 32, 2, 64, device=DEV, dtype=torch.bfloat16, block_size=16, num_blocks=2)
    cache.init_batch(2)
    with pytest.raises(AssertionError):
        cache.plan([0], [33], [0])
    cache.plan([0], [32], [0])
    with pytest.raises(BlockPoolExhaustedError):
        cache.plan([1], [1], [0])
    from nifre_b200 import Attention
    with pytest.raises(ValueError, match="layer_id is required"):
        Attention(2, 64)(torch.zeros(1, 1, 128, device=DEV), torch.zeros(1, 1, 128, device=DEV),
                         torch.zeros(1, 1, 128, device=DEV), kv_cache=cache)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("D,Hq,Hkv", [(64, 32, 8), (128, 32, 8), (64, 8, 8), (64, 16, 2), (128, 16, 16)])
def test_prefill_kernel_vs_oracle(dtype, D, Hq, Hkv):
    """Tensor-core prefill tiles (q_len >= 16) mixed with decodes and short chunks in one step."""
    past = [0, 5, 16, 300, 1000, 2048, 40, 7, 600]
    qlens = [16, 37, 64, 130, 512, 100, 1, 8, 1]
    if dtype == torch.float16 and D == 128:
        past, qlens = past[:5], qlens[:5]
    cache, g = _random_cache(Hq, Hkv, D, 16, [max(p, 1) for p in past], dtype, seed=D + Hq + Hkv, room=600)
    cache.reset_slot(0)
    T = sum(qlens)
    q = torch.randn(T, Hq * D, generator=g).to(dtype).to(DEV)
    k = torch.randn(T, Hkv * D, generator=g).to(dtype).to(DEV)
    v = torch.randn(T, Hkv * D, generator=g).to(dtype).to(DEV)
    starts = [sum(qlens[:i]) for i in range(len(qlens))]
    before = [cache.length(s) for s in range(len(qlens))]
    plan = cache.plan(list(range(len(qlens))), qlens, starts, q_heads=Hq)
    assert plan.n_tiles > 0
    cache.append_step(0, k, v, plan)
    out = torch.full_like(q, float("nan"))
    cache.attention_step(0, q, plan, out)
    kp, vp = cache.k[0].cpu(), cache.v[0].cpu()
    for s, (st, n) in enumerate(zip(starts, qlens)):
        ref = attend_paged_fp32(q[st:st + n].view(n, Hq, D).cpu(), kp, vp, cache.block_tables[s].physical_blocks(),
                                before[s] + n, Hq // Hkv, causal_base=before[s])
        torch.testing.assert_close(out[st:st + n].view(n, Hq, D).float().cpu(), ref, **_tol(dtype))
    cache.check_status()
