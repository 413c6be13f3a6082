"""The allocation-free attention entry point against the workspace one (needs a B200).

nf_paged_attention_noalloc serves callers that cannot allocate device memory
(a binding that only borrows another runtime's tensors, or a process whose
device memory is all reserved by its own pool) and so cannot pass a split-K
workspace: its scratch is a fixed buffer inside the library.  These checks run
it through the C ABI on split-K work and compare it with nf_paged_attention,
which is given a workspace owned by the cache, on two calls in a row (the
shared buffer keeps the previous call's contents, so the second call shows
that what must start at zero is cleared; a buffer filled with garbage
first shows it more strongly).  This file is collected last so
that a run stopping at its first failure has already run every other test.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"
TOL = dict(rtol=2e-2, atol=2e-2)  # the bfloat16 tolerance of the attention outputs


def _noalloc(lib, cache, q, out, plan, hq):
    from nifre_b200 import _lib
    return lib.nf_paged_attention_noalloc(
        out.data_ptr(), out.stride(0), q.data_ptr(), q.stride(0),
        cache.k[0].data_ptr(), cache.v[0].data_ptr(), _lib.dtype_code(cache.dtype),
        hq, cache.n_heads, cache.head_dim, cache.block_size, cache.num_blocks, cache.bt_dev.data_ptr(),
        cache.max_blocks_per_seq, plan.items.data_ptr(), plan.units.data_ptr(), plan.counts.data_ptr(),
        plan.n_tokens, plan.max_units, plan.split, 1.0 / cache.head_dim ** 0.5,
        cache.status.data_ptr(), _lib.stream_handle(cache.device))


def _filled_cache(ctx, hq, hkv, d, seed):
    from nifre_b200 import PagedKVCache
    g = torch.Generator().manual_seed(seed)
    cache = PagedKVCache(1, max(ctx) + 8, hkv, d, device=DEV, dtype=torch.bfloat16, block_size=16,
                         enable_prefix_cache=False)
    cache.init_batch(len(ctx))
    cache.block_allocator.set_free_order(torch.randperm(cache.num_blocks, generator=g).tolist())
    k = torch.randn(sum(ctx), hkv * d, generator=g).to(torch.bfloat16).to(DEV)
    v = torch.randn(sum(ctx), hkv * d, generator=g).to(torch.bfloat16).to(DEV)
    plan = cache.plan(list(range(len(ctx))), ctx, [sum(ctx[:i]) for i in range(len(ctx))])
    cache.append_step(0, k, v, plan)
    return cache, g


def test_noalloc_matches_workspace_entry_point_on_two_calls():
    from nifre_b200 import _lib
    lib = _lib.load()
    hq, hkv, d = 32, 8, 64
    ctx = [1, 17, 300, 513, 1000, 2049]
    cache, g = _filled_cache(ctx, hq, hkv, d, seed=11)
    B = len(ctx)
    for call in range(2):
        q = torch.randn(B, hq * d, generator=g).to(torch.bfloat16).to(DEV)
        kn = torch.randn(B, hkv * d, generator=g).to(torch.bfloat16).to(DEV)
        plan = cache.plan(list(range(B)), [1] * B, list(range(B)), split=128)  # several parts per item
        cache.append_step(0, kn, kn, plan)
        ref = torch.zeros_like(q)
        cache.attention_step(0, q, plan, ref)
        got = torch.full_like(q, float("nan"))
        rc = _noalloc(lib, cache, q, got, plan, hq)
        assert rc == 0, lib.nf_last_error().decode()
        torch.cuda.synchronize()
        assert torch.isfinite(got).all()
        torch.testing.assert_close(got.float(), ref.float(), **TOL)
    cache.check_status()


def test_noalloc_clears_a_dirty_buffer_itself():
    """Counters left nonzero in the shared buffer (filled with 0xFF: every counter -1) are cleared by the call."""
    from nifre_b200 import _lib
    lib = _lib.load()
    hq, hkv, d = 32, 8, 64
    ctx = [40, 700, 1500, 3000]
    cache, g = _filled_cache(ctx, hq, hkv, d, seed=5)
    B = len(ctx)
    stream = _lib.stream_handle(cache.device)
    for fill in (0xFF, 0x7F):
        q = torch.randn(B, hq * d, generator=g).to(torch.bfloat16).to(DEV)
        kn = torch.randn(B, hkv * d, generator=g).to(torch.bfloat16).to(DEV)
        plan = cache.plan(list(range(B)), [1] * B, list(range(B)), split=128)
        cache.append_step(0, kn, kn, plan)
        ref = torch.zeros_like(q)
        cache.attention_step(0, q, plan, ref)
        assert lib.nf_noalloc_scratch_fill(fill, stream) == 0, lib.nf_last_error().decode()
        got = torch.full_like(q, float("nan"))
        rc = _noalloc(lib, cache, q, got, plan, hq)
        assert rc == 0, lib.nf_last_error().decode()
        torch.cuda.synchronize()
        torch.testing.assert_close(got.float(), ref.float(), **TOL)
    cache.check_status()


def test_noalloc_refuses_a_plan_with_cascade_parts():
    """Cascade parts live in the caller's workspace, which this entry point does not have: flagged, out untouched."""
    import numpy as np
    from nifre_b200 import PagedKVCache, _lib
    lib = _lib.load()
    hq, hkv, d = 32, 8, 64
    rng = np.random.default_rng(3)
    g = torch.Generator().manual_seed(3)
    base = rng.integers(0, 50000, size=512).tolist()
    prompts = [base + rng.integers(0, 50000, size=20 + i).tolist() for i in range(6)]
    cache = PagedKVCache(1, 600, hkv, d, device=DEV, dtype=torch.bfloat16, block_size=16)
    cache.init_batch(len(prompts))
    for r, toks in enumerate(prompts):  # later requests import the first one's prefix blocks
        m = cache.try_load_prefix(r, toks)
        plan = cache.plan([r], [len(toks) - m], [0])
        kv = torch.randn(len(toks) - m, hkv * d, generator=g).to(torch.bfloat16).to(DEV)
        cache.append_step(0, kv, kv, plan)
        cache.register_prefix(r, toks)
    B = len(prompts)
    plan = cache.plan(list(range(B)), [1] * B, list(range(B)), q_heads=hq)
    assert plan.n_casc_tasks > 0
    kn = torch.randn(B, hkv * d, generator=g).to(torch.bfloat16).to(DEV)
    cache.append_step(0, kn, kn, plan)
    q = torch.randn(B, hq * d, generator=g).to(torch.bfloat16).to(DEV)
    sentinel = torch.full_like(q, 7.0)
    got = sentinel.clone()
    rc = _noalloc(lib, cache, q, got, plan, hq)
    assert rc == 0, lib.nf_last_error().decode()
    torch.cuda.synchronize()
    st = int(cache.status.item())
    cache.status.zero_()
    assert st == _lib.NF_STATUS_FOREIGN_PARTS
    assert torch.equal(got, sentinel)


def test_noalloc_rejects_steps_beyond_its_buffer():
    from nifre_b200 import _lib
    lib = _lib.load()
    dummy = ctypes.c_void_p(16)
    # 1M units x 32 heads x 68 floats is far beyond the built-in buffer: refused before any launch
    rc = lib.nf_paged_attention_noalloc(dummy, 2048, dummy, 2048, dummy, dummy, _lib.NF_BF16, 32, 8, 64, 16, 1,
                                        dummy, 1, dummy, dummy, dummy, 64, 1 << 20, 128, 0.125, dummy, None)
    assert rc == 1
    assert b"scratch" in lib.nf_last_error()
    # head counts whose size products would overflow 64 bits are refused as well, before any work is queued
    rc = lib.nf_paged_attention_noalloc(dummy, 2048, dummy, 2048, dummy, dummy, _lib.NF_BF16, 1 << 30, 1 << 30, 256,
                                        16, 1, dummy, 1, dummy, dummy, dummy, 1 << 30, 1 << 30, 128, 0.125, dummy, None)
    assert rc == 1
