"""Generate the golden fixtures by running the reference implementation itself.

Run from the repository root where a checkout of the reference is available,
giving its root directory (the one holding ``src/inference``) as the first
argument or in ``NIFRE_REF``:

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py <reference root>

Every fixture records inputs and the outputs of the reference's own modules
(``src/inference/attention.py``, ``paged_kv_cache.py``, ``block_allocator.py``,
``block_table.py``, ``prefix_cache.py``, ``engine.py``, ``models/gpt.py``).
The committed ``.pt`` files are what the tests read; the reference is never
read at test time.

Grouped-query cases run the reference with K/V heads repeated
(``repeat_interleave(group, dim=heads)``) because the reference has one head
count for queries and keys.
"""

from __future__ import annotations

import hashlib
import os
import random
import sys
from pathlib import Path

import torch

_root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("NIFRE_REF")
if not _root:
    raise SystemExit("usage: make_golden.py <reference root> (or set NIFRE_REF)")
REF = Path(_root) / "src"
sys.path.insert(0, str(REF))
sys.dont_write_bytecode = True

from inference.attention import Attention  # noqa: E402
from inference.backends.gpt import GptInferenceModel  # noqa: E402
from inference.block_allocator import BlockAllocator  # noqa: E402
from inference.block_table import BlockTable  # noqa: E402
from inference.engine import Engine  # noqa: E402
from inference.models.gpt import GPT_CONFIG_124M, GptModel  # noqa: E402
from inference.paged_kv_cache import PagedKVCache  # noqa: E402
from inference.prefix_cache import PrefixCache  # noqa: E402

OUT = Path(__file__).resolve().parent


def _tables(cache):
    return [t.physical_blocks() for t in cache.block_tables]


def case_smoke_paged():
    """The call sequence of the reference's attention smoke test (paged, bs 8, fp32)."""
    torch.manual_seed(0)
    H, D, L = 2, 4, 2
    attn = Attention(H, D)
    cache = PagedKVCache(num_layers=L, max_seq_len=16, n_heads=H, head_dim=D,
                         device="cpu", dtype=torch.float32, block_size=8)
    cache.init_batch(1)
    calls = []

    def run(q, k, v, input_lens=None, slots=None):
        outs = []
        for layer in range(L):
            outs.append(attn(q, k, v, kv_cache=cache, layer_id=layer,
                             input_lens=input_lens, cache_batch_indices=slots))
        calls.append(dict(q=q, k=k, v=v, input_lens=input_lens, slots=slots, outs=outs,
                          pos=cache.pos.clone(), tables=_tables(cache)))

    mk = lambda b, t: (torch.randn(b, t, H * D), torch.randn(b, t, H * D), torch.randn(b, t, H * D))
    run(*mk(1, 3))
    run(*mk(1, 1))
    pools_1 = (torch.stack(cache.k).clone(), torch.stack(cache.v).clone())
    cache.free()
    cache.init_batch(2)
    q, k, v = mk(2, 4)
    run(q, k, v, input_lens=torch.tensor([3, 4]))
    run(*mk(2, 1))
    return dict(H=H, D=D, L=L, bs=8, max_seq_len=16, calls=calls, pools_first=pools_1,
                k_final=torch.stack(cache.k).clone(), v_final=torch.stack(cache.v).clone())


def _ragged_case(seed, Hq, Hkv, D, bs, L, dtype, prompt_lens, chunk, decode_steps,
                 max_seq_len, free_shuffle=False):
    """Chunked prefill (left padded, like ModelRunner.prefill) then decode steps.

    The reference cache stores Hq heads; K/V are generated with Hkv heads and
    repeated, so the stored heads j*group..j*group+group-1 are all KV head j.
    """
    g = torch.Generator().manual_seed(seed)
    group = Hq // Hkv
    B = len(prompt_lens)
    attn = Attention(Hq, D)
    cache = PagedKVCache(num_layers=L, max_seq_len=max_seq_len, n_heads=Hq, head_dim=D,
                         device="cpu", dtype=dtype, block_size=bs, enable_prefix_cache=False)
    cache.init_batch(B)
    if free_shuffle:
        perm = torch.randperm(cache.num_blocks, generator=g).tolist()
        cache.block_allocator._free = list(perm)
    else:
        perm = None
    offsets = [0] * B
    steps = []

    def expand(x, T):
        return x.view(x.shape[0], T, Hkv, D).repeat_interleave(group, dim=2).reshape(x.shape[0], T, Hq * D)

    while any(o < n for o, n in zip(offsets, prompt_lens)):
        rows = [i for i in range(B) if offsets[i] < prompt_lens[i]]
        lens = [min(chunk, prompt_lens[i] - offsets[i]) for i in rows]
        T = max(lens)
        q = torch.randn(len(rows), T, Hq * D, generator=g).to(dtype)
        k = torch.randn(len(rows), T, Hkv * D, generator=g).to(dtype)
        v = torch.randn(len(rows), T, Hkv * D, generator=g).to(dtype)
        il = torch.tensor(lens)
        outs = [attn(q, expand(k, T), expand(v, T), kv_cache=cache, layer_id=layer,
                     input_lens=il, cache_batch_indices=rows) for layer in range(L)]
        steps.append(dict(kind="prefill", slots=rows, lens=lens, q=q, k=k, v=v, outs=outs,
                          tables=_tables(cache), pos=cache.pos.clone()))
        for i, n in zip(rows, lens):
            offsets[i] += n
    for _ in range(decode_steps):
        rows = list(range(B))
        q = torch.randn(B, 1, Hq * D, generator=g).to(dtype)
        k = torch.randn(B, 1, Hkv * D, generator=g).to(dtype)
        v = torch.randn(B, 1, Hkv * D, generator=g).to(dtype)
        outs = [attn(q, expand(k, 1), expand(v, 1), kv_cache=cache, layer_id=layer,
                     cache_batch_indices=rows) for layer in range(L)]
        steps.append(dict(kind="decode", slots=rows, lens=[1] * B, q=q, k=k, v=v, outs=outs,
                          tables=_tables(cache), pos=cache.pos.clone()))
    # stored pools keep only one of each group of repeated heads
    k_pool = torch.stack(cache.k)[:, :, :, ::group].clone()
    v_pool = torch.stack(cache.v)[:, :, :, ::group].clone()
    return dict(seed=seed, Hq=Hq, Hkv=Hkv, D=D, bs=bs, L=L, dtype=str(dtype), prompt_lens=prompt_lens,
                chunk=chunk, decode_steps=decode_steps, max_seq_len=max_seq_len, steps=steps,
                free_order=perm, num_blocks=cache.num_blocks, k_pool=k_pool, v_pool=v_pool)


def case_allocator_semantics():
    """Block ids produced by the reference cache under allocate/reset/prefix reuse."""
    log = []
    cache = PagedKVCache(num_layers=2, max_seq_len=64, n_heads=2, head_dim=4, device="cpu",
                         dtype=torch.float32, block_size=4, enable_prefix_cache=True)
    cache.init_batch(3)
    key = torch.zeros(9, 2, 4)
    for layer in range(2):
        cache.append(0, layer, key, key)
    log.append(("append0_9", _tables(cache), cache.allocated_blocks))
    for layer in range(2):
        cache.append(1, layer, key[:5], key[:5])
    log.append(("append1_5", _tables(cache), cache.allocated_blocks))
    cache.register_prefix(0, list(range(9)))
    log.append(("register0", _tables(cache), cache.allocated_blocks))
    cache.reset_slot(0)
    log.append(("reset0", _tables(cache), cache.allocated_blocks))
    n = cache.try_load_prefix(2, list(range(8)) + [77, 78])
    log.append(("load2", _tables(cache), cache.allocated_blocks, n))
    for layer in range(2):
        cache.append(2, layer, key[:3], key[:3])
    log.append(("append2_3", _tables(cache), cache.allocated_blocks))
    cache.reset_slot(1)
    for layer in range(2):
        cache.append(0, layer, key[:6], key[:6])
    log.append(("append0_6", _tables(cache), cache.allocated_blocks))
    # small prefix cache forcing LRU eviction
    alloc = BlockAllocator(6)
    pc = PrefixCache(alloc, block_size=2, max_entries=2)
    t = BlockTable(alloc, 2)
    t.ensure_capacity(6)
    pc.insert([1, 2, 3, 4, 5, 6], t.physical_blocks())
    evict = dict(blocks=t.physical_blocks(), refc=[alloc.refcount(b) for b in range(6)],
                 entries=len(pc.entries), lookup=pc.lookup([1, 2, 3, 4, 5, 6]),
                 lookup_tail=pc.lookup([5, 6]))
    t.clear()
    evict["after_clear_free"] = alloc.free_count
    return dict(log=log, evict=evict)


def _gpt_param_digest(model):
    return {n: (tuple(p.shape), hashlib.sha256(p.detach().contiguous().numpy().tobytes()).hexdigest())
            for n, p in model.state_dict().items()}


class _MarginModel:
    """Wraps the reference model and records the smallest top-1/top-2 logit gap."""

    def __init__(self, inner):
        self.inner = inner
        self.config = inner.config
        self.min_margin = float("inf")

    @property
    def dtype(self):
        return self.inner.dtype

    def eval(self):
        self.inner.eval()

    def __call__(self, token_ids, kv_cache=None, input_lens=None, cache_batch_indices=None):
        logits = self.inner(token_ids, kv_cache=kv_cache, input_lens=input_lens,
                            cache_batch_indices=cache_batch_indices)
        top = logits[:, -1, :].topk(2, dim=-1).values
        self.min_margin = min(self.min_margin, float((top[:, 0] - top[:, 1]).min()))
        return logits


def case_gpt_engine(num_layers, emb, heads, ctx, n_prompts, lo, hi, new_tokens, chunk, slots, seed=0):
    cfg = dict(GPT_CONFIG_124M)
    cfg.update(num_layers=num_layers, emb_dim=emb, num_heads=heads, context_length=ctx)
    torch.manual_seed(seed)
    model = GptModel(cfg).eval()
    digest = _gpt_param_digest(model)
    wrapped = _MarginModel(GptInferenceModel(model))
    eng = Engine(wrapped, max_concurrent_requests=slots, device=torch.device("cpu"),
                 prefill_chunk_size=chunk, max_tokens_per_step=2048)
    rng = random.Random(seed)
    prompts = []
    for _ in range(n_prompts):
        n = rng.randint(lo, hi)
        prompts.append([rng.randrange(cfg["vocab_size"]) for _ in range(n)])
    ids = [eng.add_request(p, new_tokens) for p in prompts]
    steps = 0
    while eng.step():
        steps += 1
    done = eng.get_completed()
    tokens = [done[i].output_token_ids for i in ids]
    return dict(cfg=cfg, seed=seed, prompts=prompts, tokens=tokens, steps=steps, chunk=chunk,
                slots=slots, num_blocks=eng.cache.num_blocks, min_margin=wrapped.min_margin,
                digest=digest)


def main():
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    fx = {}
    fx["smoke_paged"] = case_smoke_paged()
    fx["mha_fp32"] = _ragged_case(1, Hq=4, Hkv=4, D=16, bs=4, L=2, dtype=torch.float32,
                                  prompt_lens=[5, 9, 3], chunk=4, decode_steps=6, max_seq_len=64)
    fx["gqa_bf16"] = _ragged_case(2, Hq=8, Hkv=2, D=64, bs=16, L=1, dtype=torch.bfloat16,
                                  prompt_lens=[40, 17, 70, 33], chunk=32, decode_steps=5,
                                  max_seq_len=128, free_shuffle=True)
    fx["gqa_fp32"] = _ragged_case(3, Hq=16, Hkv=4, D=64, bs=16, L=1, dtype=torch.float32,
                                  prompt_lens=[21, 16, 37], chunk=16, decode_steps=3,
                                  max_seq_len=64, free_shuffle=True)
    fx["gqa_d128_bf16"] = _ragged_case(4, Hq=16, Hkv=4, D=128, bs=16, L=1, dtype=torch.bfloat16,
                                       prompt_lens=[33, 20], chunk=24, decode_steps=2,
                                       max_seq_len=64, free_shuffle=True)
    fx["allocator"] = case_allocator_semantics()
    torch.save(fx, OUT / "paged_attention_golden.pt")

    eng = {}
    eng["tiny"] = case_gpt_engine(2, 32, 4, 64, n_prompts=3, lo=3, hi=20, new_tokens=5, chunk=4, slots=2)
    eng["gpt124m_cfg1"] = case_gpt_engine(12, 768, 12, 2048, n_prompts=8, lo=32, hi=256,
                                         new_tokens=64, chunk=128, slots=8)
    torch.save(eng, OUT / "engine_golden.pt")
    for name in ("paged_attention_golden.pt", "engine_golden.pt"):
        print(name, (OUT / name).stat().st_size, "bytes")
    print("cfg1 min top1-top2 margin", eng["gpt124m_cfg1"]["min_margin"], "steps", eng["gpt124m_cfg1"]["steps"])


if __name__ == "__main__":
    main()
