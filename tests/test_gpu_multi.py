"""The KV-head-sharded path on two B200s: the attention kernels' own gathered output (peer stores over NVLink).

Two processes, one per GPU, each hold half of the KV heads (and their query
heads) of the same batch; the block tables, positions and schedule are the
same on both (the same seeds).  ``PagedKVCache.attention_step(...,
exchange=PeerExchange)`` makes the decode and prefill kernels store every
output row into both ranks' gathered buffers and end with a signal-and-wait,
replacing attention + an NCCL all-gather.  Checked on every rank:

* the gathered output of a decode step, of a mixed step (prefill chunks on the
  tensor-core kernel plus decodes) and of a prefill-only step (the
  stand-alone barrier) equals float32 attention over the full heads
  (rtol = atol = 2e-2, the bf16 tolerance) -- the reference's attention
  (attention.py:106-152) with grouped-query heads expanded;
* both ranks end with bit-identical gathered buffers;
* a CUDA graph of an exchanging decode launch, replayed three times, gives
  the eager launch's gathered rows (the exchange's epoch lives on the device);
* a rank that skips an exchange makes the other rank's kernel give up after
  its time limit with NF_STATUS_WAIT_TIMEOUT set (a wait nothing satisfies;
  nothing faults), after which the context still answers.

Skipped with fewer than two GPUs.  NVLS is off in NCCL (which only swaps
the IPC handles and runs barriers here).
"""

import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

WORLD = 2
TOL = dict(rtol=2e-2, atol=2e-2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _expected(q, kfull, vfull, hq, hkv, d, causal_base=None):
    """float32 attention of q (n, hq, d) over keys kfull/vfull (m, hkv, d) with causal masking of the last n."""
    g = hq // hkv
    n, m = q.shape[0], kfull.shape[0]
    K = kfull.float().repeat_interleave(g, dim=1).transpose(0, 1)
    V = vfull.float().repeat_interleave(g, dim=1).transpose(0, 1)
    s = (q.float().transpose(0, 1) @ K.transpose(1, 2)) / d ** 0.5
    base = m - n if causal_base is None else causal_base
    mask = torch.arange(m).unsqueeze(0) > (torch.arange(n) + base).unsqueeze(1)
    s.masked_fill_(mask, float("-inf"))
    return (s.softmax(-1) @ V).transpose(0, 1).reshape(n, hq * d)


def _worker(rank, port, out_q):
    import datetime

    import torch.distributed as dist

    from nifre_b200 import PagedKVCache, _lib
    from nifre_b200.sharding import HeadShard, PeerExchange

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    res = {"rank": rank, "errors": []}
    try:
        Hq, Hkv, D, bs = 32, 8, 64, 16
        shard = HeadShard(WORLD, rank, Hq, Hkv, D)
        hq, hkv = shard.q_heads, shard.kv_heads
        kvc = shard.kv_columns()
        qc = shard.q_columns()
        g = torch.Generator().manual_seed(0)
        rng = np.random.default_rng(0)
        ctx = rng.integers(100, 3000, size=14).tolist() + [0, 0]  # two empty slots for prefill chunks
        B = len(ctx)
        cache = PagedKVCache(1, 4096, hkv, D, device=dev, dtype=torch.bfloat16, block_size=bs,
                             enable_prefix_cache=False)
        cache.init_batch(B)
        cache.block_allocator.set_free_order(torch.randperm(cache.num_blocks, generator=g).tolist())
        # every rank draws the full K/V and keeps its heads' columns
        hist_k = [torch.randn(c, Hkv * D, generator=g).to(torch.bfloat16) for c in ctx]
        hist_v = [torch.randn(c, Hkv * D, generator=g).to(torch.bfloat16) for c in ctx]
        fill = [i for i in range(B) if ctx[i]]
        kf = torch.cat([hist_k[i] for i in fill])[:, kvc].contiguous().to(dev)
        vf = torch.cat([hist_v[i] for i in fill])[:, kvc].contiguous().to(dev)
        plan = cache.plan(fill, [ctx[i] for i in fill], np.cumsum([0] + [ctx[i] for i in fill][:-1]).tolist())
        cache.append_step(0, kf, vf, plan)
        ex = PeerExchange(shard, 512, torch.bfloat16, dev, slots=3)

        def run_step(slots, q_lens, slot_buf, skip=False):
            T = sum(q_lens)
            starts = np.cumsum([0] + q_lens[:-1]).tolist()
            q = torch.randn(T, Hq * D, generator=g).to(torch.bfloat16)
            k = torch.randn(T, Hkv * D, generator=g).to(torch.bfloat16)
            v = torch.randn(T, Hkv * D, generator=g).to(torch.bfloat16)
            p = cache.plan(slots, q_lens, starts, q_heads=hq)
            cache.append_step(0, k[:, kvc].contiguous().to(dev), v[:, kvc].contiguous().to(dev), p)
            if skip:  # this rank leaves the exchange out: the peer's wait must run out
                return None
            out = ex.out(slot_buf, T)
            cache.attention_step(0, q[:, qc].contiguous().to(dev), p, out, exchange=ex)
            torch.cuda.synchronize(dev)
            cache.check_status()
            got = ex.gathered(slot_buf, T).float().cpu()
            worst = 0.0
            for i, s in enumerate(slots):
                n, st = q_lens[i], starts[i]
                hist_k[s] = torch.cat([hist_k[s], k[st:st + n]])
                hist_v[s] = torch.cat([hist_v[s], v[st:st + n]])
                exp = _expected(q[st:st + n].view(n, Hq, D), hist_k[s].view(-1, Hkv, D), hist_v[s].view(-1, Hkv, D),
                                Hq, Hkv, D)
                torch.testing.assert_close(got[st:st + n], exp, **TOL)
                worst = max(worst, float((got[st:st + n] - exp).abs().max()))
            # both ranks hold the same gathered rows, bit for bit
            mine = ex.gathered(slot_buf, T).contiguous()
            both = [torch.empty_like(mine) for _ in range(WORLD)]
            dist.all_gather(both, mine)
            assert all(torch.equal(both[0], b) for b in both)
            return worst

        dec = list(range(14))
        res["decode"] = run_step(dec, [1] * 14, 0)
        res["mixed"] = run_step([14] + dec[:6], [96] + [1] * 6, 1)       # one chunk on the prefill kernel
        res["prefill_only"] = run_step([15], [64], 2)                     # stand-alone barrier
        res["second_decode"] = run_step(dec, [1] * 14, 0)                 # buffer 0 again, next epoch
        # a CUDA graph of an exchanging launch: the epoch lives on the device, so replays exchange afresh
        T = 14
        qg = torch.randn(T, Hq * D, generator=g).to(torch.bfloat16)
        kg = torch.randn(T, Hkv * D, generator=g).to(torch.bfloat16)
        pg = cache.plan(dec, [1] * T, list(range(T)), q_heads=hq)
        cache.append_step(0, kg[:, kvc].contiguous().to(dev), kg[:, kvc].contiguous().to(dev), pg)
        qd = qg[:, qc].contiguous().to(dev)
        og = ex.out(2, T)
        cache.attention_step(0, qd, pg, og, exchange=ex)
        torch.cuda.synchronize(dev)
        ref = ex.gathered(2, T).clone()
        ex.gathered(2, T).zero_()
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(side):
            with torch.cuda.graph(graph, stream=side):
                cache.attention_step(0, qd, pg, og, exchange=ex)
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize(dev)
        cache.check_status()
        res["graph_equal"] = bool(torch.equal(ex.gathered(2, T), ref))
        del graph
        # failure detection: rank 1 leaves one exchange out; rank 0's kernel gives up after its limit
        if rank == 1:
            run_step(dec, [1] * 14, 1, skip=True)
        else:
            T = 14
            q = torch.randn(T, Hq * D, generator=g).to(torch.bfloat16)
            kk = torch.randn(T, Hkv * D, generator=g).to(torch.bfloat16)
            p = cache.plan(dec, [1] * T, list(range(T)), q_heads=hq)
            cache.append_step(0, kk[:, kvc].contiguous().to(dev), kk[:, kvc].contiguous().to(dev), p)
            cache.attention_step(0, q[:, qc].contiguous().to(dev), p, ex.out(1, T), exchange=ex)
            torch.cuda.synchronize(dev)
            st = int(cache.status.item())
            cache.status.zero_()
            res["timeout_status"] = st
            res["context_ok"] = bool(torch.ones(4, device=dev).sum().item() == 4.0)
        dist.barrier()
        ex.close()
    except Exception as e:  # noqa: BLE001 -- reported to the parent
        import traceback
        res["errors"].append(traceback.format_exc())
    finally:
        out_q.put(res)
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs two GPUs")
def test_sharded_gathered_output_two_gpus():
    import torch.multiprocessing as mp

    from nifre_b200 import _lib

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = [q.get(timeout=600) for _ in procs]
    for p in procs:
        p.join(timeout=120)
    for r in results:
        assert not r["errors"], r["errors"][0]
    r0 = next(r for r in results if r["rank"] == 0)
    for key in ("decode", "mixed", "prefill_only", "second_decode"):
        assert r0[key] is not None and r0[key] < 2e-2
    assert all(r["graph_equal"] for r in results)
    assert r0["timeout_status"] & _lib.NF_STATUS_WAIT_TIMEOUT
    assert r0["context_ok"]
