"""The allocation-free attention entry point against the workspace one (needs a B200).

nf_paged_attention_noalloc serves callers that cannot allocate device memory
(a binding that only borrows another runtime's tensors, or a process whose
device memory is all reserved by its own pool) and so cannot pass a split-K
workspace: its scratch is a fixed buffer inside the library.  These checks run
it through the C ABI on split-K work and compare it with nf_paged_attention,
which is given a workspace owned by the cache, on two calls in a row (the
shared buffer keeps the previous call's contents, so the second call shows
that what must start at zero is cleared).  This file is collected last so
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


def test_noalloc_rejects_steps_beyond_its_buffer():
    from nifre_b200 import _lib
    lib = _lib.load()
    dummy = ctypes.c_void_p(16)
    # 1M units x 32 heads x 68 floats is far beyond the built-in buffer: refused before any launch
    rc = lib.nf_paged_attention_noalloc(dummy, 2048, dummy, 2048, dummy, dummy, _lib.NF_BF16, 32, 8, 64, 16, 1,
                                        dummy, 1, dummy, dummy, dummy, 64, 1 << 20, 128, 0.125, dummy, None)
    assert rc == 1
    assert b"scratch" in lib.nf_last_error()
