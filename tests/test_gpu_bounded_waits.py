"""Failure detection on the device: every wait of the kernels gives up after a time limit.

The pipeline waits of the attention, prefill and cascade kernels (mbarrier
waits) and the end-of-launch wait of the split-K kernels (a grid counter) are
bounded: when the limit runs out the wait sets NF_STATUS_WAIT_TIMEOUT and
returns false, and the kernel leaves its loops instead of spinning forever.
``nf_selftest_wait`` runs those same wait functions with a short limit on a
wait that nothing satisfies (an mbarrier no thread arrives on, a counter
nothing increments).  The tests check that the kernel ends, the status bit is
set, the wait reports failure, and the context stays usable for a normal
attention step afterwards.  Nothing faults, traps or hangs.
"""

import pytest
import torch

from nifre_b200 import _lib

DEV = "cuda"
LIMIT = 2_000_000  # SM cycles: about a millisecond


def _run(kind, counter=None, target=1):
    lib = _lib.load()
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    result = torch.full((1,), -1, dtype=torch.int32, device=DEV)
    rc = lib.nf_selftest_wait(kind, LIMIT, None if counter is None else counter.data_ptr(), target,
                              status.data_ptr(), result.data_ptr(), _lib.stream_handle(torch.device(DEV)))
    assert rc == 0, lib.nf_last_error().decode()
    torch.cuda.synchronize()
    return int(status.item()), int(result.item())


def test_selftest_wait_argument_errors():
    """Refused on the host before any launch (no GPU needed)."""
    lib = _lib.load()
    assert lib.nf_selftest_wait(2, LIMIT, None, 1, None, None, None) == 1
    assert lib.nf_selftest_wait(0, 0, None, 1, None, None, None) == 1
    assert lib.nf_selftest_wait(0, 1 << 40, None, 1, None, None, None) == 1
    assert b"limit" in lib.nf_last_error()


@pytest.mark.gpu
def test_mbarrier_wait_gives_up():
    st, res = _run(0)
    assert st == _lib.NF_STATUS_WAIT_TIMEOUT
    assert res == 0


@pytest.mark.gpu
def test_grid_counter_wait_gives_up_and_succeeds_when_reached():
    counter = torch.zeros(1, dtype=torch.int32, device=DEV)  # nothing increments it
    st, res = _run(1, counter, target=1)
    assert st == _lib.NF_STATUS_WAIT_TIMEOUT and res == 0
    counter.fill_(3)  # already at the target: the wait returns at once, no flag
    st, res = _run(1, counter, target=3)
    assert st == 0 and res == 1


@pytest.mark.gpu
def test_context_usable_after_timeouts():
    """After waits have run out, a normal paged-attention step still runs and matches the oracle."""
    from nifre_b200 import PagedKVCache
    from oracle.attention import attend_paged_fp32
    _run(0)
    _run(1, torch.zeros(1, dtype=torch.int32, device=DEV))
    hq, hkv, d = 8, 2, 64
    ctx = [5, 130, 600]
    g = torch.Generator().manual_seed(0)
    cache = PagedKVCache(1, 700, hkv, d, device=DEV, dtype=torch.bfloat16, block_size=16,
                         enable_prefix_cache=False)
    cache.init_batch(len(ctx))
    kv = torch.randn(sum(ctx), hkv * d, generator=g).to(torch.bfloat16).to(DEV)
    plan = cache.plan([0, 1, 2], ctx, [0, ctx[0], ctx[0] + ctx[1]])
    cache.append_step(0, kv, kv, plan)
    q = torch.randn(3, hq * d, generator=g).to(torch.bfloat16).to(DEV)
    kn = torch.randn(3, hkv * d, generator=g).to(torch.bfloat16).to(DEV)
    plan = cache.plan([0, 1, 2], [1, 1, 1], [0, 1, 2], split=64)
    cache.append_step(0, kn, kn, plan)
    out = torch.zeros_like(q)
    cache.attention_step(0, q, plan, out)
    torch.cuda.synchronize()
    cache.check_status()
    for s in range(3):
        ref = attend_paged_fp32(q[s].view(1, hq, d).cpu(), cache.k[0].cpu(), cache.v[0].cpu(),
                                cache.block_tables[s].physical_blocks(), ctx[s] + 1, hq // hkv)
        torch.testing.assert_close(out[s].view(hq, d).float().cpu(), ref[0], rtol=2e-2, atol=2e-2)
