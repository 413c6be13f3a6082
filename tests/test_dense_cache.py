"""The dense per-row KVCache (nifre ``src/inference/kv_cache.py:4-79``) on the paged kernels.

Host checks run on the CPU; the rest (marked gpu) compare the storage
bit-exactly with what was appended, the attention outputs with the oracle
(bfloat16 within rtol/atol 2e-2, float32 within rtol 1e-4 / atol 1e-5) and
the engine's greedy tokens on the dense cache with the reference Engine's
recorded tokens.
"""

import pytest
import torch

from oracle.attention import attend_paged_fp32

DEV = "cuda"


def _tol(dtype):
    return dict(rtol=1e-4, atol=1e-5) if dtype == torch.float32 else dict(rtol=2e-2, atol=2e-2)


def test_dense_cache_host_contract():
    """Constructor and attributes of kv_cache.py:12-22; no device path without CUDA."""
    from nifre_b200 import KVCache, PagedKVCache, _lib
    from nifre_b200.batching import make_kv_cache
    from nifre_b200.data_model import ModelConfig
    c = KVCache(3, 100, 4, 64, device="cpu", dtype=torch.bfloat16)
    assert isinstance(c, PagedKVCache)
    assert (c.num_layers, c.max_seq_len, c.n_heads, c.head_dim, c.dtype) == (3, 100, 4, 64, torch.bfloat16)
    assert c.batch_size == 0 and c.pos is None and c.k is None and c.v is None
    assert c.block_size == 100 and c.prefix_cache is None
    with pytest.raises(_lib.NifreError):
        c.init_batch(2)
    cfg = ModelConfig(num_layers=2, max_seq_len=64, n_heads=4, head_dim=16, vocab_size=10, pad_token_id=0)
    m = make_kv_cache(cfg, "cpu")
    assert isinstance(m, KVCache) and m.dtype == torch.float16 and m.max_seq_len == 64 and m.n_heads == 4


@pytest.mark.gpu
def test_dense_cache_storage_and_cursor():
    """(B, max_seq_len, H, D) tensors per layer; pos advances after the last layer; get views; reset keeps rows."""
    from nifre_b200 import Attention, KVCache
    g = torch.Generator().manual_seed(11)
    L, S, H, D = 2, 48, 4, 64
    cache = KVCache(L, S, H, D, device=DEV, dtype=torch.bfloat16)
    cache.init_batch(3)
    assert all(t.shape == (3, S, H, D) for t in cache.k + cache.v)
    assert cache.allocated_blocks == 3
    attn = Attention(H, D)
    B, T = 3, 9
    lens = [9, 4, 1]  # left-padded prefill rows
    qkv = [torch.randn(B, T, H * D, generator=g).to(torch.bfloat16).to(DEV) for _ in range(3 * L)]
    for layer in range(L):
        q, k, v = qkv[3 * layer:3 * layer + 3]
        out = attn(q, k, v, kv_cache=cache, layer_id=layer, input_lens=lens)
        assert out.shape == q.shape
        for b, n in enumerate(lens):
            assert torch.count_nonzero(out[b, : T - n]) == 0  # pad rows stay zero (attention.py:79)
        if layer < L - 1:
            assert cache.lengths().tolist() == [0, 0, 0]  # pos moves after the last layer only
    assert cache.lengths().tolist() == lens
    for layer in range(L):
        k, v = qkv[3 * layer + 1], qkv[3 * layer + 2]
        for b, n in enumerate(lens):
            kk, vv = cache.get(b, layer)
            assert kk.data_ptr() == cache.k[layer][b].data_ptr()  # a view of row b
            assert torch.equal(kk.reshape(n, -1), k[b, T - n:])
            assert torch.equal(vv.reshape(n, -1), v[b, T - n:])
            assert torch.equal(cache.k[layer][b, :n].reshape(n, -1), k[b, T - n:])
    cache.reset_slot(1)
    assert cache.length(1) == 0 and cache.allocated_blocks == 3
    assert cache.get(1, 0)[0].shape == (0, H, D)
    cache.check_status()


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("max_seq_len", [512, 100])
def test_dense_cache_attention_vs_oracle(dtype, max_seq_len):
    """Prefill chunks continuing cached rows plus decodes, one plan: rows of max_seq_len tokens
    (512: tensor-map decode and tensor-core prefill; 100, not a multiple of 16: the per-warp decode)."""
    from nifre_b200 import KVCache
    g = torch.Generator().manual_seed(13)
    Hq, Hkv, D = 16, 4, 64
    cache = KVCache(1, max_seq_len, Hkv, D, device=DEV, dtype=dtype)
    cache.init_batch(4)
    first = [30, 1, 60, 17]
    steps = [first, [37, 1, 20, 1]]
    for qlens in steps:
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
            assert cache.block_tables[s].physical_blocks() == [s]
            ref = attend_paged_fp32(q[st:st + n].view(n, Hq, D).cpu(), cache.k[0].cpu(), cache.v[0].cpu(), [s],
                                    before[s] + n, Hq // Hkv, causal_base=before[s])
            torch.testing.assert_close(out[st:st + n].view(n, Hq, D).float().cpu(), ref, **_tol(dtype))
    cache.check_status()


@pytest.mark.gpu
def test_dense_cache_full_row_rejected():
    """Appending past max_seq_len fails on the host before any launch (kv_cache.py:52)."""
    from nifre_b200 import KVCache
    cache = KVCache(1, 32, 2, 64, device=DEV, dtype=torch.bfloat16)
    cache.init_batch(2)
    k = torch.zeros(33, 128, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(AssertionError):
        cache.append(0, 0, k.view(33, 2, 64), k.view(33, 2, 64))
    assert cache.length(0) == 0


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["tiny", "gpt124m_cfg1"])
def test_engine_dense_cache_greedy_tokens(golden_engine, name):
    """Engine(use_paged_kv_cache=False) runs on KVCache and gives the reference's greedy tokens."""
    from nifre_b200 import Engine, GptInferenceModel, GptModel, KVCache
    case = golden_engine[name]
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.manual_seed(case["seed"])
    model = GptModel(case["cfg"]).eval().to("cuda")
    eng = Engine(GptInferenceModel(model), max_concurrent_requests=case["slots"], device="cuda",
                 prefill_chunk_size=case["chunk"], max_tokens_per_step=2048, use_paged_kv_cache=False)
    new_tokens = len(case["tokens"][0])
    ids = [eng.add_request(p, new_tokens) for p in case["prompts"]]
    while eng.step():
        pass
    assert isinstance(eng.cache, KVCache)
    done = eng.get_completed()
    assert [done[i].output_token_ids for i in ids] == case["tokens"]
    eng.cache.check_status()
