"""KV-head sharding host logic on CPU with world size 2 (gloo).

Each rank computes plain attention on its own heads (torch, CPU: the host
logic under test is the head split and the output exchange, not the kernel)
and all-gathers; the result must equal the unsharded computation on every
rank.  Also: a rank that raises before the exchange makes the other rank's
collective fail within the process-group timeout instead of hanging.
"""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from nifre_b200.sharding import HeadShard


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _attend(q, k, v, hq, hkv, d):
    rows = q.shape[0]
    qh = q.view(rows, hq, d).transpose(0, 1)
    kh = k.view(rows, hkv, d).transpose(0, 1).repeat_interleave(hq // hkv, 0)
    vh = v.view(rows, hkv, d).transpose(0, 1).repeat_interleave(hq // hkv, 0)
    s = qh @ kh.transpose(1, 2) / d ** 0.5
    s = s.masked_fill(torch.triu(torch.ones(rows, rows, dtype=torch.bool), 1), float("-inf"))
    return (s.softmax(-1) @ vh).transpose(0, 1).reshape(rows, hq * d)


def _worker(rank, world, port, mode, result):
    import datetime

    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    try:
        hq, hkv, d, rows = 8, 4, 16, 10
        g = torch.Generator().manual_seed(0)
        q = torch.randn(rows, hq * d, generator=g)
        k = torch.randn(rows, hkv * d, generator=g)
        v = torch.randn(rows, hkv * d, generator=g)
        shard = HeadShard(world, rank, hq, hkv, d)
        if mode == "fail" and rank == 1:
            raise RuntimeError("rank 1 fails before the exchange")
        ql, kl, vl = shard.local(q, k, v)
        out_local = _attend(ql, kl, vl, shard.q_heads, shard.kv_heads, d)
        try:
            full = shard.gather(out_local)
        except Exception as exc:  # the peer never joined: the collective ends with an error
            result[rank] = ("error", type(exc).__name__)
            return
        ref = _attend(q, k, v, hq, hkv, d)
        result[rank] = ("ok", float((full - ref).abs().max()))
    except RuntimeError as exc:
        result[rank] = ("raised", str(exc))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(mode):
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        result = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, result)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=120)
        for p in procs:
            if p.is_alive():
                p.kill()
        return dict(result)


def test_head_shard_gather_matches_unsharded():
    res = _run("ok")
    assert set(res) == {0, 1}
    for rank in (0, 1):
        status, err = res[rank]
        assert status == "ok" and err < 1e-5


def test_failed_rank_ends_peer_collective_with_error():
    res = _run("fail")
    assert res[1][0] == "raised"
    assert res[0][0] == "error"


def test_head_shard_ranges():
    s = HeadShard(4, 3, 32, 8, 64)
    assert (s.kv_heads, s.q_heads) == (2, 8)
    assert s.q_columns() == slice(3 * 8 * 64, 4 * 8 * 64) and s.kv_columns() == slice(3 * 2 * 64, 4 * 2 * 64)
    with pytest.raises(ValueError):
        HeadShard(3, 0, 32, 8, 64)
