"""The QKV projection fused with the KV append (nf_qkv_append, tcgen05).

Reference: GptAttention.forward (src/inference/models/gpt.py:38-51) projects
q, k and v with three nn.Linear layers and the cache appends k and v
(paged_kv_cache.py:107-121).  Checked here:

* q and the pool rows of the step's tokens against the float32 product
  x W^T (+ b), rounded once to bfloat16/half (rtol = atol = 1e-2: one rounding
  of values of order 1), on a ragged step over a randomly permuted pool;
* the scatter is exact: the pool rows equal, bit for bit, the k/v rows the
  same kernel writes into a dense buffer with the identity slot mapping, and
  no other pool row changes;
* pos advances on the last layer only, as the reference's append does;
* a bfloat16 GPT through the engine gives the same prefill tokens with the
  fused projection as with cuBLAS + nf_kv_append, and at least 95% of the
  decode tokens (the two GEMMs round their fp32 sums differently).
"""

import numpy as np
import pytest
import torch

DEV = "cuda"


def _step(hq, hkv, d, lens, dtype, seed, layers=1):
    from nifre_b200 import PagedKVCache
    g = torch.Generator().manual_seed(seed)
    cache = PagedKVCache(layers, 512, hkv, d, device=DEV, dtype=dtype, block_size=16, enable_prefix_cache=False)
    cache.init_batch(len(lens))
    cache.block_allocator.set_free_order(torch.randperm(cache.num_blocks, generator=g).tolist())
    plan = cache.plan(list(range(len(lens))), lens, np.cumsum([0] + lens[:-1]).tolist(), q_heads=hq)
    return cache, plan, g


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("hq,hkv,d,kdim,bias", [(32, 8, 64, 2048, False), (12, 12, 64, 768, True),
                                                 (8, 2, 128, 1000, True)])
def test_qkv_append_vs_float32(dtype, hq, hkv, d, kdim, bias):
    from nifre_b200 import _lib
    lens = [1, 37, 130, 1, 200, 5]
    cache, plan, g = _step(hq, hkv, d, lens, dtype, seed=hq + kdim)
    T, nq, nkv = sum(lens), hq * d, hkv * d
    x = torch.randn(T, kdim, generator=g).to(dtype).to(DEV)
    w = (torch.randn(nq + 2 * nkv, kdim, generator=g) / kdim ** 0.5).to(dtype).to(DEV)
    b = torch.randn(nq + 2 * nkv, generator=g).to(dtype).to(DEV) if bias else None
    k_before, v_before = cache.k[0].clone(), cache.v[0].clone()
    q = torch.empty(T, nq, dtype=dtype, device=DEV)
    cache.project_append_step(0, x, w, b, plan, q)
    torch.cuda.synchronize()
    cache.check_status()
    ref = x.float() @ w.float().T + (b.float() if bias else 0.0)
    tol = dict(rtol=1e-2, atol=1e-2)
    torch.testing.assert_close(q.float(), ref[:, :nq], **tol)
    slots = plan.slot_mapping.long()
    kp, vp = cache.k[0].view(-1, nkv), cache.v[0].view(-1, nkv)
    torch.testing.assert_close(kp[slots].float(), ref[:, nq:nq + nkv], **tol)
    torch.testing.assert_close(vp[slots].float(), ref[:, nq + nkv:], **tol)
    # the scatter is exact: the same kernel into a dense buffer with slot t = row t
    dense_k = torch.zeros(T, nkv, dtype=dtype, device=DEV)
    dense_v = torch.zeros_like(dense_k)
    q2 = torch.empty_like(q)
    ident = torch.arange(T, dtype=torch.int32, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    lib = _lib.load()
    _lib.check(lib.nf_qkv_append(x.data_ptr(), kdim, T, w.data_ptr(), b.data_ptr() if bias else None, kdim, nq, nkv,
                                 q2.data_ptr(), nq, dense_k.data_ptr(), dense_v.data_ptr(), T, _lib.dtype_code(dtype),
                                 ident.data_ptr(), None, 0, None, status.data_ptr(),
                                 _lib.stream_handle(torch.device(DEV))), "nf_qkv_append")
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert torch.equal(q2, q)
    assert torch.equal(kp[slots], dense_k) and torch.equal(vp[slots], dense_v)
    # no other pool row changed (compared as bit patterns: unwritten pool memory may hold NaNs)
    other = torch.ones(kp.shape[0], dtype=torch.bool, device=DEV)
    other[slots] = False
    bits = torch.int16
    assert torch.equal(kp[other].view(bits), k_before.view(-1, nkv)[other].view(bits))
    assert torch.equal(vp[other].view(bits), v_before.view(-1, nkv)[other].view(bits))


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("rows", [1, 33, 64, 100, 128])
@pytest.mark.parametrize("hq,hkv,d,kdim,bias", [(32, 8, 64, 2048, False), (2, 1, 64, 256, True),
                                                 (8, 2, 128, 1024, True)])
def test_qkv_few_rows_vs_float32(dtype, rows, hq, hkv, d, kdim, bias):
    """Decode-sized steps (1 to 128 rows, one 128-row tile with its zero-filled tail): q and the pool rows
    against the float32 product, one rounding (rtol = atol = 1e-2), and bit-equal to the same rows written
    into a dense buffer (the scatter); (2, 1, 64): output tiles on both sides of the k/v boundary."""
    from nifre_b200 import _lib
    lens = [1] * rows  # decode rows
    cache, plan, g = _step(hq, hkv, d, lens, dtype, seed=rows + kdim)
    T, nq, nkv = rows, hq * d, hkv * d
    x = torch.randn(T, kdim, generator=g).to(dtype).to(DEV)
    w = (torch.randn(nq + 2 * nkv, kdim, generator=g) / kdim ** 0.5).to(dtype).to(DEV)
    b = torch.randn(nq + 2 * nkv, generator=g).to(dtype).to(DEV) if bias else None
    q = torch.empty(T, nq, dtype=dtype, device=DEV)
    cache.project_append_step(0, x, w, b, plan, q)
    torch.cuda.synchronize()
    cache.check_status()
    ref = x.float() @ w.float().T + (b.float() if bias else 0.0)
    tol = dict(rtol=1e-2, atol=1e-2)
    torch.testing.assert_close(q.float(), ref[:, :nq], **tol)
    slots = plan.slot_mapping.long()
    kp, vp = cache.k[0].view(-1, nkv), cache.v[0].view(-1, nkv)
    torch.testing.assert_close(kp[slots].float(), ref[:, nq:nq + nkv], **tol)
    torch.testing.assert_close(vp[slots].float(), ref[:, nq + nkv:], **tol)
    dense_k = torch.zeros(T, nkv, dtype=dtype, device=DEV)
    dense_v = torch.zeros_like(dense_k)
    q2 = torch.empty_like(q)
    ident = torch.arange(T, dtype=torch.int32, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    lib = _lib.load()
    _lib.check(lib.nf_qkv_append(x.data_ptr(), kdim, T, w.data_ptr(), b.data_ptr() if bias else None, kdim, nq, nkv,
                                 q2.data_ptr(), nq, dense_k.data_ptr(), dense_v.data_ptr(), T, _lib.dtype_code(dtype),
                                 ident.data_ptr(), None, 0, None, status.data_ptr(),
                                 _lib.stream_handle(torch.device(DEV))), "nf_qkv_append")
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert torch.equal(q2, q)
    assert torch.equal(kp[slots], dense_k) and torch.equal(vp[slots], dense_v)


@pytest.mark.gpu
def test_qkv_append_advances_pos_on_last_layer_only():
    lens = [3, 1, 20]
    cache, plan, g = _step(8, 2, 64, lens, torch.bfloat16, seed=1, layers=2)
    T, nq, nkv, kdim = sum(lens), 8 * 64, 2 * 64, 256
    x = torch.randn(T, kdim, generator=g).to(torch.bfloat16).to(DEV)
    w = (torch.randn(nq + 2 * nkv, kdim, generator=g) / 16).to(torch.bfloat16).to(DEV)
    q = torch.empty(T, nq, dtype=torch.bfloat16, device=DEV)
    cache.project_append_step(0, x, w, None, plan, q)
    torch.cuda.synchronize()
    assert cache.pos.cpu().tolist() == [0, 0, 0] and not plan.closed
    cache.project_append_step(1, x, w, None, plan, q)
    torch.cuda.synchronize()
    assert cache.pos.cpu().tolist() == lens and plan.closed
    assert [cache.length(s) for s in range(3)] == lens


@pytest.mark.gpu
def test_engine_bf16_fused_projection_matches_cublas_path():
    import random

    from nifre_b200 import Engine, GptInferenceModel, GptModel
    from nifre_b200.gpt import TransformerBlock
    cfg = dict(vocab_size=1000, context_length=512, emb_dim=256, num_heads=4, num_layers=2, drop_rate=0.0,
               qkv_bias=True)
    rnd = random.Random(7)
    prompts = [[rnd.randrange(1000) for _ in range(rnd.randint(20, 120))] for _ in range(5)]
    runs = []
    try:
        for fused in (True, False):
            TransformerBlock.fused_projection = fused
            torch.manual_seed(0)
            model = GptModel(cfg).eval().to("cuda", dtype=torch.bfloat16)
            with torch.no_grad():
                model.out_head.weight.mul_(30.0)  # well separated logits: argmax ties out of reach of rounding
            eng = Engine(GptInferenceModel(model), max_concurrent_requests=5, device="cuda", prefill_chunk_size=64)
            ids = [eng.add_request(p, 16) for p in prompts]
            while eng.step():
                pass
            done = eng.get_completed()
            runs.append([done[i].output_token_ids for i in ids])
            eng.cache.check_status()
    finally:
        TransformerBlock.fused_projection = True
    fused_out, plain_out = runs
    assert [t[0] for t in fused_out] == [t[0] for t in plain_out]
    pairs = [(a, b) for x, y in zip(fused_out, plain_out) for a, b in zip(x[1:], y[1:])]
    assert sum(a == b for a, b in pairs) >= 0.95 * len(pairs)


def test_qkv_append_argument_errors():
    """Refused on the host before any launch (no GPU needed)."""
    import ctypes

    from nifre_b200 import _lib
    lib = _lib.load()
    d = ctypes.c_void_p(256)
    # float32 operands, widths not multiples of 64, unaligned rows
    assert lib.nf_qkv_append(d, 64, 4, d, None, 64, 64, 64, d, 64, d, d, 16, _lib.NF_F32, d, None, 0, None, d,
                             None) == 3
    assert lib.nf_qkv_append(d, 64, 4, d, None, 64, 96, 64, d, 64, d, d, 16, _lib.NF_BF16, d, None, 0, None, d,
                             None) == 3
    assert lib.nf_qkv_append(d, 63, 4, d, None, 64, 64, 64, d, 64, d, d, 16, _lib.NF_BF16, d, None, 0, None, d,
                             None) == 1
    assert b"aligned" in lib.nf_last_error()
