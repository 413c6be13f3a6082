"""Cascade attention over shared prefix blocks: grouping on the host (CPU) and parity (B200).

Decode sequences that imported the same prefix blocks (``try_load_prefix``,
nifre ``src/inference/paged_kv_cache.py:87-105``) have those keys attended
once per group by ``nf_cascade_attention``; the decode launch covers the
rest and merges.  The result must be the same attention as without the
cascade: bfloat16 within rtol/atol 2e-2 of the float32 oracle over each
sequence's own block table.
"""

import numpy as np
import pytest
import torch

from oracle.attention import attend_paged_fp32

DEV = "cuda"
TOL = dict(rtol=2e-2, atol=2e-2)


def _host_cache(tables, ctx, bs=16, hkv=8):
    """A PagedKVCache with host state only (block tables and positions), for the planning logic."""
    from nifre_b200 import BlockAllocator, BlockTable, PagedKVCache
    c = PagedKVCache(1, 4096, hkv, 64, device="cpu", dtype=torch.bfloat16, block_size=bs)
    n = 1 + max(max(t) for t in tables)
    c.block_allocator = BlockAllocator(n)
    c.block_tables = []
    for t in tables:
        bt = BlockTable(c.block_allocator, bs)
        bt._physical_blocks = list(t)
        c.block_tables.append(bt)
    c.pos_host = np.asarray(ctx, dtype=np.int64)
    c._sm_count = 148
    return c


def test_cascade_groups_host():
    """Groups = decode sequences sharing leading blocks, cut to <= 128 / G sequences; shared keys = common blocks."""
    bs = 16
    pre_a = list(range(0, 64))          # 1024-key prefix
    pre_b = list(range(100, 104))       # 64 keys: the minimum
    tables, ctx = [], []
    for i in range(40):                 # 40 sequences on prefix A (32 + 8 with G = 4)
        tables.append(pre_a + [1000 + 2 * i, 1001 + 2 * i])
        ctx.append(len(pre_a) * bs + 20)
    tables.append(pre_a[:10] + [2000, 2001])  # diverges after 10 blocks: shortens A's common run
    ctx.append(10 * bs + 5)
    for i in range(2):
        tables.append(pre_b + [3000 + i])
        ctx.append(len(pre_b) * bs + 3)
    tables.append([4000, 4001])         # alone: no cascade
    ctx.append(20)
    c = _host_cache(tables, ctx, bs)
    c.cascade_limits = lambda group: (128, 256, False)  # the mma.sync kernel's task sizes
    S = len(tables)
    slots = np.arange(S)
    q_lens = np.ones(S, dtype=np.int64)
    q_starts = np.arange(S, dtype=np.int64) * 3 + 5  # rows of the queries in q
    dec = np.ones(S, dtype=bool)
    shared, nparts, tasks, toks = c._cascade_groups(slots, q_lens, q_starts, np.asarray(ctx), dec, 4)
    # prefix A: 41 members whose common run is 10 blocks -> groups of 32 and 9
    assert shared[:41].tolist() == [160] * 41
    assert shared[41:43].tolist() == [64, 64] and shared[43] == 0
    groups = sorted({(t[0], t[1], t[2]) for t in tasks}, key=lambda g: g[1])
    assert [g[2] for g in groups] == [32, 9, 2]
    assert sorted(t for t, _ in toks) == list(range(43))
    assert all(row == q_starts[t] for t, row in toks)
    # CASCADE_WAVES x 148 SMs / 8 KV heads = 37 ranges wanted, in proportion to the shared keys; runs this
    # short give one 16-key tile per range (10 + 10 + 4)
    assert len(tasks) == 24
    for slot, first, count in groups:
        members = [t for t, _ in toks[first:first + count]]
        assert slot == members[0]
        mine = [t for t in tasks if t[1] == first]
        assert [t[3] for t in mine] == list(range(len(mine)))
        assert mine[0][4] == 0 and mine[-1][5] == shared[members[0]]
        assert all(a[5] == b[4] for a, b in zip(mine, mine[1:]))  # contiguous key ranges
        assert all(t[4] % 16 == 0 and t[5] % 16 == 0 and 16 <= t[5] - t[4] <= c.CASCADE_MAX_KEYS for t in mine)
        assert max(t[5] - t[4] for t in mine) - min(t[5] - t[4] for t in mine) <= 16  # near-equal ranges
        assert all(nparts[m] == len(mine) for m in members)
    # sequences with more than one new token are never grouped
    q2 = q_lens.copy()
    q2[:] = 2
    assert c._cascade_groups(slots, q2, q_starts, np.asarray(ctx), dec, 4)[2] == []
    # with G = 8, at most 16 sequences per group
    tasks8 = c._cascade_groups(slots, q_lens, q_starts, np.asarray(ctx), dec, 8)[2]
    assert max(t[2] for t in tasks8) == 16
    # a long shared run is cut into ranges of at most CASCADE_MAX_KEYS keys
    long_c = _host_cache([list(range(200)) + [900 + i] for i in range(4)], [200 * bs + 7] * 4, bs)
    long_c.cascade_limits = c.cascade_limits
    lt = long_c._cascade_groups(np.arange(4), np.ones(4, np.int64), np.arange(4), np.full(4, 200 * bs + 7),
                                np.ones(4, bool), 4)[2]
    assert len(lt) == 37 and max(t[5] - t[4] for t in lt) <= 256  # 37 ranges of 5-6 tiles
    # the next decode step of the same batch reuses the grouping; a replaced table or a position moved
    # back under a shared run recomputes it
    again = c._cascade_groups(slots, q_lens, q_starts, np.asarray(ctx) + 1, dec, 8)
    assert again is c._cascade_groups(slots, q_lens, q_starts, np.asarray(ctx) + 2, dec, 8)
    assert c._cascade_groups(slots, q_lens, q_starts, np.asarray(ctx) - 1000, dec, 8) is not again
    c.block_tables[3].epoch += 1
    assert c._cascade_groups(slots, q_lens, q_starts, np.asarray(ctx), dec, 8) is not again


def test_cascade_limits_and_tensor_core_groups_host():
    """nf_cascade_limits: 256 query rows and any key count on the tensor-core path (16-bit pools, D 64/128,
    G in {1, 2, 4, 8}), 128 rows and 256 keys on the mma.sync kernel; tensor-core tasks aim at one item per
    SM with at least CASCADE_TC_MIN_KEYS keys each."""
    bs = 16
    c = _host_cache([[0]], [1], bs)
    assert c.cascade_limits(4) == (256, 1 << 30, True)
    assert c.cascade_limits(8) == (256, 1 << 30, True)
    assert c.cascade_limits(3) == (128, 256, False)
    assert c.cascade_limits(16) == (128, 256, False)
    # 70 sequences on a 2048-key prefix, G = 4: groups of at most 64; 148 SMs / 8 KV heads = 18 items wanted
    tables = [list(range(128)) + [500 + i] for i in range(70)]
    ctx = [128 * bs + 9] * 70
    c = _host_cache(tables, ctx, bs)
    S = len(tables)
    shared, nparts, tasks, toks = c._cascade_groups(np.arange(S), np.ones(S, np.int64), np.arange(S),
                                                    np.asarray(ctx), np.ones(S, bool), 4)
    groups = sorted({(t[1], t[2]) for t in tasks})
    assert [n for _, n in groups] == [64, 6]
    assert shared.tolist() == [2048] * 70
    for first, n in groups:
        mine = [t for t in tasks if t[1] == first]
        assert mine[0][4] == 0 and mine[-1][5] == 2048 and all(a[5] == b[4] for a, b in zip(mine, mine[1:]))
        assert all(t[5] - t[4] >= c.CASCADE_TC_MIN_KEYS for t in mine)
    assert len(tasks) == 16  # 9 parts each, at most 2048 / 256 = 8


def _shared_prefix_cache(hq, hkv, D, prefixes, n_per, suffix, dtype, seed, tail_div=None):
    """Requests importing shared prompt prefixes the way the engine does (try_load_prefix, prefill the rest,
    register_prefix), each with its own random suffix; ``tail_div`` requests diverge inside the prefix."""
    from nifre_b200 import PagedKVCache
    rng = np.random.default_rng(seed)
    g = torch.Generator().manual_seed(seed)
    prompts = []
    for p in prefixes:
        base = rng.integers(0, 50000, size=p).tolist()
        for j in range(n_per):
            prompts.append(base + rng.integers(0, 50000, size=int(rng.integers(*suffix))).tolist())
    if tail_div:
        for r in range(0, len(prompts), tail_div):
            cut = len(prompts[r]) // 3
            prompts[r] = prompts[r][:cut] + rng.integers(0, 50000, size=len(prompts[r]) - cut).tolist()
    B = len(prompts)
    cache = PagedKVCache(1, max(len(p) for p in prompts) + 8, hkv, D, device=DEV, dtype=dtype, block_size=16)
    cache.init_batch(B)
    for r, toks in enumerate(prompts):
        m = cache.try_load_prefix(r, toks)
        n = len(toks) - m
        plan = cache.plan([r], [n], [0])
        k = torch.randn(n, hkv * D, generator=g).to(dtype).to(DEV)
        v = torch.randn(n, hkv * D, generator=g).to(dtype).to(DEV)
        cache.append_step(0, k, v, plan)
        cache.register_prefix(r, toks)
    return cache, g


@pytest.mark.gpu
@pytest.mark.parametrize("D,hq,hkv", [(64, 32, 8), (128, 32, 8), (64, 8, 8), (64, 16, 2),  # tensor cores
                                       (64, 4, 1), (128, 4, 1),  # one KV head (an 8-way shard): one-head decode
                                       (64, 24, 8), (128, 12, 2)])  # G = 3 and 6: the mma.sync kernel
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_cascade_decode_vs_oracle(D, hq, hkv, dtype):
    """A decode step over shared prefixes: cascade + decode merge equals the oracle per sequence."""
    cache, g = _shared_prefix_cache(hq, hkv, D, [256, 512, 48], 12, (1, 90), dtype, seed=D + hq,
                                    tail_div=7)
    B = cache.batch_size
    before = [cache.length(s) for s in range(B)]
    plan = cache.plan(list(range(B)), [1] * B, list(range(B)), q_heads=hq)
    assert plan.n_casc_tasks > 0 and (plan.shared_keys > 0).sum() >= 2 * 2
    q = torch.randn(B, hq * D, generator=g).to(dtype).to(DEV)
    k = torch.randn(B, hkv * D, generator=g).to(dtype).to(DEV)
    v = torch.randn(B, hkv * D, generator=g).to(dtype).to(DEV)
    cache.append_step(0, k, v, plan)
    out = torch.zeros_like(q)
    cache.attention_step(0, q, plan, out)
    cache.check_status()
    kp, vp = cache.k[0].cpu(), cache.v[0].cpu()
    for b in range(B):
        ref = attend_paged_fp32(q[b].view(1, hq, D).cpu(), kp, vp, cache.block_tables[b].physical_blocks(),
                                before[b] + 1, hq // hkv)
        torch.testing.assert_close(out[b].view(hq, D).float().cpu(), ref[0], **TOL)


@pytest.mark.gpu
def test_cascade_matches_plain_decode_and_many_groups():
    """Same step with and without the cascade (two caches built alike): outputs agree; 40 sequences on one
    prefix with G = 4 make one group (the tensor-core path takes 256 / G = 64 per group); a long prefix gives
    several key ranges per group."""
    outs = []
    for casc in (True, False):
        cache, g = _shared_prefix_cache(32, 8, 64, [2048], 40, (1, 40), torch.bfloat16, seed=5)
        cache.enable_cascade = casc
        B = cache.batch_size
        plan = cache.plan(list(range(B)), [1] * B, list(range(B)), q_heads=32)
        assert (plan.n_casc_tasks > 0) == casc
        if casc:
            tasks = plan.casc_tasks.view(-1, 8).cpu().numpy()
            assert sorted({(int(t[1]), int(t[2])) for t in tasks}) == [(0, 40)]
            assert plan.n_casc_tasks > 2
        q = torch.randn(B, 32 * 64, generator=g).to(torch.bfloat16).to(DEV)
        k = torch.randn(B, 8 * 64, generator=g).to(torch.bfloat16).to(DEV)
        v = torch.randn(B, 8 * 64, generator=g).to(torch.bfloat16).to(DEV)
        cache.append_step(0, k, v, plan)
        out = torch.zeros_like(q)
        cache.attention_step(0, q, plan, out)
        cache.check_status()
        outs.append(out.float().cpu())
    torch.testing.assert_close(outs[0], outs[1], **TOL)


@pytest.mark.gpu
@pytest.mark.parametrize("n_per,suffix,cross", [(40, (1, 60), False), (60, (1, 700), True)])
def test_cascade_single_own_unit_vs_oracle(n_per, suffix, cross):
    """Enough decode sequences on shared prefixes that each one whose own keys fit in one unit gets one: the
    decode kernel merges its cascade parts in that unit's epilogue (unit records: parts in the low 16 bits of
    the last field, units in the high bits).  With longer sequences too (cross), their items have several
    units, and the last of them to finish merges every part.  Oracle per sequence."""
    cache, g = _shared_prefix_cache(32, 8, 64, [256, 512], n_per, suffix, torch.bfloat16, seed=11 + int(cross))
    B = cache.batch_size
    before = [cache.length(s) for s in range(B)]
    plan = cache.plan(list(range(B)), [1] * B, list(range(B)), q_heads=32)
    assert plan.n_casc_tasks > 0
    units = plan.units.view(-1, 8)[:plan.decode_units].cpu().numpy()
    single = ((units[:, 7] >> 16) == 1) & ((units[:, 7] & 0xFFFF) > 1)
    assert single.sum() >= 40
    flags = int(plan.counts[2].item())
    assert bool(flags & 2) == cross and flags & 1
    q = torch.randn(B, 32 * 64, generator=g).to(torch.bfloat16).to(DEV)
    k = torch.randn(B, 8 * 64, generator=g).to(torch.bfloat16).to(DEV)
    cache.append_step(0, k, k, plan)
    out = torch.zeros_like(q)
    cache.attention_step(0, q, plan, out)
    cache.check_status()
    kp, vp = cache.k[0].cpu(), cache.v[0].cpu()
    for b in range(B):
        ref = attend_paged_fp32(q[b].view(1, 32, 64).cpu(), kp, vp, cache.block_tables[b].physical_blocks(),
                                before[b] + 1, 4)
        torch.testing.assert_close(out[b].view(32, 64).float().cpu(), ref[0], **TOL)


@pytest.mark.gpu
def test_cascade_bad_task_flagged():
    """A task naming more queries than there are records is flagged on the status word and writes nothing."""
    from nifre_b200 import _lib
    cache, g = _shared_prefix_cache(32, 8, 64, [256], 4, (1, 20), torch.bfloat16, seed=9)
    B = cache.batch_size
    plan = cache.plan(list(range(B)), [1] * B, list(range(B)), q_heads=32)
    assert plan.n_casc_tasks > 0
    lib = _lib.load()
    ws = torch.zeros(plan.max_units * 32 * 68, dtype=torch.float32, device=DEV)
    bad = torch.tensor([0, 0, 1000, 0, 0, 64, 0, 0], dtype=torch.int32, device=DEV)  # more queries than records
    q = torch.zeros(B, 32 * 64, dtype=torch.bfloat16, device=DEV)
    _lib.check(lib.nf_cascade_attention(
        ws.data_ptr(), ws.numel(), q.data_ptr(), q.stride(0), q.shape[0], cache.k[0].data_ptr(), cache.v[0].data_ptr(),
        _lib.NF_BF16, 32, 8, 64, 16, cache.num_blocks, cache.bt_dev.data_ptr(), cache.max_blocks_per_seq,
        plan.items.data_ptr(), plan.counts.data_ptr(), B, plan.max_units, bad.data_ptr(), 1,
        plan.casc_toks.data_ptr(), plan.n_casc_toks, 0.125,
        cache.status.data_ptr(), _lib.stream_handle(cache.device)), "nf_cascade_attention")
    torch.cuda.synchronize()
    assert int(cache.status.item()) == _lib.NF_STATUS_BAD_SHARED
    assert int(torch.count_nonzero(ws)) == 0
    cache.status.zero_()


@pytest.mark.gpu
def test_cascade_across_steps_and_mixed_step():
    """Several decode steps in a row (the grouping memoised, contexts crossing block boundaries, two layers),
    then one step mixing prefill chunks with the cascaded decodes; every output checked against the oracle."""
    from nifre_b200 import PagedKVCache
    hq, hkv, D, L = 32, 8, 64, 2
    rng = np.random.default_rng(21)
    g = torch.Generator().manual_seed(21)
    base = rng.integers(0, 50000, size=300).tolist()
    prompts = [base + rng.integers(0, 50000, size=int(rng.integers(1, 30))).tolist() for _ in range(10)]
    extra = [rng.integers(0, 50000, size=int(n)).tolist() for n in (200, 40)]  # later prefills
    B = len(prompts) + len(extra)
    cache = PagedKVCache(L, 700, hkv, D, device=DEV, dtype=torch.bfloat16, block_size=16)
    cache.init_batch(B)
    for r, toks in enumerate(prompts):
        m = cache.try_load_prefix(r, toks)
        n = len(toks) - m
        plan = cache.plan([r], [n], [0])
        for layer in range(L):
            cache.append_step(layer, torch.randn(n, hkv * D, generator=g).to(torch.bfloat16).to(DEV),
                              torch.randn(n, hkv * D, generator=g).to(torch.bfloat16).to(DEV), plan)
        cache.register_prefix(r, toks)

    def check(slots, q_lens, q, out, before, layer):
        kp, vp = cache.k[layer].cpu(), cache.v[layer].cpu()
        row = 0
        for s, n in zip(slots, q_lens):
            ref = attend_paged_fp32(q[row:row + n].view(n, hq, D).cpu(), kp, vp, cache.block_tables[s].physical_blocks(),
                                    before[s] + n, hq // hkv, causal_base=before[s])
            torch.testing.assert_close(out[row:row + n].view(n, hq, D).float().cpu(), ref, **TOL)
            row += n

    dec = list(range(len(prompts)))
    for step in range(20):  # 20 steps: every sequence crosses at least one block boundary
        before = {s: cache.length(s) for s in dec}
        plan = cache.plan(dec, [1] * len(dec), dec, q_heads=hq)
        assert plan.n_casc_tasks > 0
        for layer in range(L):
            q = torch.randn(len(dec), hq * D, generator=g).to(torch.bfloat16).to(DEV)
            k = torch.randn(len(dec), hkv * D, generator=g).to(torch.bfloat16).to(DEV)
            v = torch.randn(len(dec), hkv * D, generator=g).to(torch.bfloat16).to(DEV)
            cache.append_step(layer, k, v, plan)
            out = torch.zeros_like(q)
            cache.attention_step(layer, q, plan, out)
            if step % 6 == 0 or step == 19:
                check(dec, [1] * len(dec), q, out, before, layer)
    # mixed: two prefill chunks (new slots) first, then the decodes, in one plan
    slots = [len(prompts), len(prompts) + 1] + dec
    q_lens = [len(extra[0]), len(extra[1])] + [1] * len(dec)
    starts = np.concatenate([[0], np.cumsum(q_lens)[:-1]]).tolist()
    before = {s: cache.length(s) for s in slots}
    plan = cache.plan(slots, q_lens, starts, q_heads=hq)
    assert plan.n_tiles > 0 and plan.n_casc_tasks > 0
    T = sum(q_lens)
    for layer in range(L):
        q = torch.randn(T, hq * D, generator=g).to(torch.bfloat16).to(DEV)
        k = torch.randn(T, hkv * D, generator=g).to(torch.bfloat16).to(DEV)
        v = torch.randn(T, hkv * D, generator=g).to(torch.bfloat16).to(DEV)
        cache.append_step(layer, k, v, plan)
        out = torch.zeros_like(q)
        cache.attention_step(layer, q, plan, out)
        check(slots, q_lens, q, out, before, layer)
    cache.check_status()
