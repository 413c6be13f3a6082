"""Host-side logic and the C ABI surface (CPU only, no kernel launches).

The allocator / block table / prefix cache checks follow the reference's own
tests (tests/test_block_allocator.py, test_block_table.py, test_prefix_cache.py
of jyotilakra92/nifre) and compare allocation order with the oracle.
"""

import ctypes
import random
import re
from pathlib import Path

import pytest

from nifre_b200.block_allocator import BlockAllocator, BlockPoolExhaustedError
from nifre_b200.block_table import BlockTable
from nifre_b200.prefix_cache import PrefixCache
from oracle.paged import OracleAllocator, OraclePrefixIndex, OracleTable

ROOT = Path(__file__).resolve().parent.parent


# ---------------------------------------------------------------- allocator
def test_allocator_errors_and_counts():
    with pytest.raises(ValueError, match="num_blocks must be positive"):
        BlockAllocator(0)
    a = BlockAllocator(4)
    blocks = a.allocate_many(2)
    assert blocks == [3, 2]
    assert (a.allocated_count, a.free_count, a.utilization) == (2, 2, 0.5)
    a.free_many(blocks)
    assert (a.allocated_count, a.free_count) == (0, 4)
    with pytest.raises(ValueError, match="count must be positive"):
        a.allocate_many(0)
    with pytest.raises(ValueError, match="out of range"):
        a.free(99)
    b = a.allocate()
    a.free(b)
    with pytest.raises(ValueError, match="not allocated"):
        a.free(b)
    x, y = a.allocate(), a.allocate()
    with pytest.raises(ValueError, match="duplicate"):
        a.free_many([x, x])
    one = BlockAllocator(1)
    one.allocate()
    with pytest.raises(BlockPoolExhaustedError, match="only 0 free"):
        one.allocate_many(1)
    a.free_many([])


def test_allocator_reuse_and_refcount():
    a = BlockAllocator(2)
    first = a.allocate()
    a.free(first)
    assert a.allocate() == first
    a.retain(first)
    assert a.refcount(first) == 2
    a.release(first)
    assert a.allocated_count == 1
    a.release(first)
    assert a.allocated_count == 0 and a.free_count == 2
    with pytest.raises(ValueError, match="not allocated"):
        a.retain(0)


def test_allocator_matches_oracle_random_ops():
    rng = random.Random(0)
    n = 64
    ours, ref = BlockAllocator(n), OracleAllocator(n)
    perm = list(range(n))
    rng.shuffle(perm)
    ours.set_free_order(perm)
    ref.free = list(perm)
    live = []
    for _ in range(2000):
        op = rng.random()
        if op < 0.5 and ours.free_count:
            k = rng.randint(1, min(5, ours.free_count))
            got = ours.allocate_many(k)
            exp = [ref.allocate() for _ in range(k)]
            assert got == exp
            live += got
        elif op < 0.7 and live:
            b = rng.choice(live)
            ours.retain(b)
            ref.retain(b)
            live.append(b)
        elif live:
            b = live.pop(rng.randrange(len(live)))
            ours.release(b)
            ref.release(b)
        assert ours.free_ids() == ref.free


# ---------------------------------------------------------------- block table
def test_block_table_semantics():
    with pytest.raises(ValueError, match="block_size must be positive"):
        BlockTable(BlockAllocator(4), 0)
    t = BlockTable(BlockAllocator(8), 16)
    t.ensure_capacity(0)
    assert t.physical_blocks() == []
    t.ensure_capacity(5)
    blocks = t.physical_blocks()
    t.ensure_capacity(5)
    assert t.physical_blocks() == blocks
    t.ensure_capacity(17)
    assert len(t.physical_blocks()) == 2
    assert t.resolve(0) == (t.physical_blocks()[0], 0)
    assert t.resolve(16) == (t.physical_blocks()[1], 0)
    assert t.resolve(9) == (t.physical_blocks()[0], 9)
    with pytest.raises(IndexError, match="no allocated block"):
        t.resolve(32)
    with pytest.raises(ValueError, match="total_tokens must be non-negative"):
        t.ensure_capacity(-1)


def test_block_table_import_clear_exhaust():
    a = BlockAllocator(4)
    t = BlockTable(a, 4)
    b = a.allocate()
    t.import_blocks([b])
    assert a.refcount(b) == 2
    e0 = t.epoch
    t.clear()
    assert t.epoch != e0 and a.refcount(b) == 1
    t2 = BlockTable(a, 4)
    t2.ensure_capacity(4)
    with pytest.raises(ValueError, match="non-empty"):
        t2.import_blocks([0])
    small = BlockTable(BlockAllocator(1), 1)
    small.ensure_capacity(1)
    with pytest.raises(BlockPoolExhaustedError):
        small.ensure_capacity(2)


def test_block_table_partial_allocation_on_exhaustion_matches_reference():
    """The reference allocates one block at a time and keeps what it got before failing."""
    a = BlockAllocator(3)
    t = BlockTable(a, 2)
    with pytest.raises(BlockPoolExhaustedError, match="need 1 blocks, only 0 free"):
        t.ensure_capacity(10)
    ra = OracleAllocator(3)
    rt = OracleTable(ra, 2)
    with pytest.raises(Exception):
        rt.ensure(10)
    assert t.physical_blocks() == rt.blocks


# ---------------------------------------------------------------- prefix cache
def test_prefix_cache_matches_oracle():
    rng = random.Random(1)
    for trial in range(20):
        a, ra = BlockAllocator(64), OracleAllocator(64)
        pc, rpc = PrefixCache(a, 4, max_entries=6), OraclePrefixIndex(ra, 4, max_entries=6)
        for _ in range(30):
            toks = [rng.randrange(3) for _ in range(rng.randint(1, 14))]
            if rng.random() < 0.5:
                assert pc.lookup(toks) == rpc.lookup(toks)
            else:
                n = len(toks) // 4
                if a.free_count < n:
                    continue
                blocks = a.allocate_many(n) if n else []
                for _ in range(n):
                    ra.allocate()
                pc.insert(toks, blocks)
                rpc.insert(toks, blocks)
            assert a.free_ids() == ra.free
            assert list(pc.entries.items()) == list(rpc.entries.items())


def test_prefix_cache_validation_and_snapshot():
    a = BlockAllocator(2)
    with pytest.raises(ValueError, match="block_size must be positive"):
        PrefixCache(a, 0)
    with pytest.raises(ValueError, match="max_entries must be positive"):
        PrefixCache(a, 4, max_entries=0)
    pc = PrefixCache(a, 2)
    b = a.allocate()
    pc.insert([1, 2], [b])
    pc.insert([1, 2], [b])
    assert a.refcount(b) == 2
    assert pc.lookup([1, 2, 3]) == (2, [b])
    assert pc.snapshot()["hits"] == 1


# ---------------------------------------------------------------- C ABI surface
def _declared_symbols():
    text = (ROOT / "include" / "nifre_b200.h").read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\*?\s+\*?(nf_\w+)\s*\(", text, re.M)))


def test_library_exports_every_declared_symbol():
    from nifre_b200 import _lib
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    syms = _declared_symbols()
    assert set(syms) >= {"nf_pack_step", "nf_kv_append", "nf_paged_attention", "nf_attention_workspace",
                         "nf_last_error", "nf_abi_version", "nf_cascade_attention"}
    for s in syms:
        assert hasattr(lib, s), s
    assert set(_lib.EXPORTS) <= set(syms)
    assert _lib.load().nf_abi_version() == 14


def test_workspace_sizing_and_argument_errors():
    """Host-side checks of the C ABI (no device work is done by these calls)."""
    from nifre_b200 import _lib
    import torch
    pf, ci = _lib.workspace_sizes(100, 64, 32, 8, 64, torch.bfloat16)
    assert pf == 100 * 32 * 68 and ci == 64 * 8 + 4  # (acc, m, l, pad) per part; counters + work queue
    pf, ci = _lib.workspace_sizes(10, 4, 8, 1, 128, torch.bfloat16)
    assert pf == 10 * 8 * 132 and ci == 4 + 4
    with pytest.raises(_lib.NifreError, match="multiple of num_kv_heads"):
        _lib.workspace_sizes(1, 1, 6, 4, 64, torch.bfloat16)
    with pytest.raises(_lib.NifreError, match="more than 8"):
        _lib.workspace_sizes(1, 1, 64, 4, 64, torch.bfloat16)
    lib = _lib.load()
    rc = lib.nf_kv_append(None, None, 0, 0, None, None, 0, 0, 0, None, None, 0, 1, 1, None, 0, None, None, None)
    assert rc == 1 and b"n_tokens" in lib.nf_last_error()


def test_seq_unit_sizes_policy():
    """The shortest sequences holding one wave of keys get quarter-size units; small steps none."""
    import numpy as np
    from nifre_b200.paged_kv_cache import seq_unit_sizes
    rng = np.random.default_rng(0)
    keys = rng.integers(500, 4000, size=64)
    split, sms = 256, 148
    small = seq_unit_sizes(keys[:4], split, sms)
    assert (small == split).all()
    sizes = seq_unit_sizes(keys, split, sms)
    fine = sizes < split
    assert set(sizes.tolist()) == {split, split // 4}
    wave = sms * split
    assert keys[fine].sum() >= wave
    assert keys[fine].max() <= keys[~fine].min()  # the shortest ones
    assert keys[fine].sum() - keys[fine].max() < wave  # and no more than needed
    assert (seq_unit_sizes(keys, 32, sms) >= 16).all()


def test_prefill_order_covers_items_longest_first():
    """The prefill queue order: every (tile, KV head) item once, by decreasing key tiles."""
    import numpy as np
    from nifre_b200.paged_kv_cache import _prefill_order
    rng = np.random.default_rng(0)
    tiles = [(0, 64 * t, 64, int(p) + 64 * t) for t, p in enumerate(rng.integers(0, 2048, size=60))]
    H = 8
    order = _prefill_order(tiles, H)
    assert order.dtype == np.int32
    assert sorted(order.tolist()) == list(range(len(tiles) * H))
    cost = [(p + n + 127) // 128 + 1 for (_, _, n, p) in tiles]
    c = [cost[i // H] for i in order.tolist()]
    assert all(a >= b for a, b in zip(c, c[1:]))


def test_split_for_policy():
    """Unit sizes: multiples of 128 sized per resident decode CTA for the tensor-map kernel; multiples of 32
    sized per resident warp for the per-warp kernel (float32 pools), so small batches spread over the GPU."""
    import torch

    from nifre_b200 import PagedKVCache
    bf = PagedKVCache(1, 4096, 8, 64, device="cpu", dtype=torch.bfloat16, block_size=16)
    bf._sm_count = 148
    assert bf.decode_workers == 148  # one CTA per SM covers the 8 KV heads
    assert bf.split_for(64 * 2000) == 256 and bf.split_for(100) == 128
    assert all(bf.split_for(n) % 128 == 0 for n in (1, 10_000, 1_000_000, 10_000_000))
    shard = PagedKVCache(1, 4096, 1, 64, device="cpu", dtype=torch.bfloat16, block_size=16)
    shard._sm_count = 148
    assert shard.decode_workers == 148 * 8  # one KV head per CTA: eight smaller CTAs per SM
    f32 = PagedKVCache(1, 4096, 12, 64, device="cpu", dtype=torch.float32, block_size=16)
    f32._sm_count = 148
    assert f32.split_for(8 * 300) == 32  # 8 sequences x 12 heads: 32-key units
    big = f32.split_for(64 * 4000)
    assert big % 32 == 0 and big > 32


def test_attention_refuses_dtypes_other_than_the_cache_dtype():
    """The reference attends in q's dtype with new K/V at projection precision (attention.py:121-133); the
    library attends in the cache dtype, so q/k/v of another dtype are refused on the host, before any launch."""
    import torch
    from nifre_b200 import Attention, PagedKVCache
    cache = PagedKVCache(1, 64, 2, 64, device="cpu", dtype=torch.float16)
    attn = Attention(4, 64)
    q = torch.zeros(1, 1, 256)
    kv = torch.zeros(1, 1, 128)
    with pytest.raises(ValueError, match="must equal the cache dtype"):
        attn(q, kv, kv, kv_cache=cache, layer_id=0)
    with pytest.raises(ValueError, match="must equal the cache dtype"):
        attn(q.half(), kv, kv.half(), kv_cache=cache, layer_id=0)


def test_argument_structs_match_the_header(tmp_path):
    """The ctypes mirrors of NfGather / NfAttentionArgs / NfAppendArgs have the C layout (sizes and offsets)."""
    import ctypes
    import shutil
    import subprocess

    from nifre_b200 import _lib
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    structs = {"NfGather": _lib.NfGather, "NfAttentionArgs": _lib.NfAttentionArgs, "NfAppendArgs": _lib.NfAppendArgs}
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "nifre_b200.h"', 'int main(void) {']
    for name, cls in structs.items():
        lines.append(f'  printf("{name} size %zu\\n", sizeof({name}));')
        for field, _ in cls._fields_:
            lines.append(f'  printf("{name} {field} %zu\\n", offsetof({name}, {field}));')
    lines.append("  return 0;\n}")
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.check_call([cc, "-I", str(ROOT / "include"), str(src), "-o", str(exe)])
    got = {}
    for line in subprocess.check_output([str(exe)], text=True).splitlines():
        name, field, val = line.split()
        got[(name, field)] = int(val)
    for name, cls in structs.items():
        assert got[(name, "size")] == ctypes.sizeof(cls), name
        for field, _ in cls._fields_:
            assert got[(name, field)] == getattr(cls, field).offset, (name, field)
