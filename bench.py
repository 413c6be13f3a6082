#!/usr/bin/env python
"""Benchmark of the ragged paged-attention decode path on B200.

Workload (default): Llama-3.2-1B-shaped paged decode, bfloat16 -- 16 layers,
32 query heads, 8 KV heads, head_dim 64, block size 16, 64 sequences with
context lengths uniform in [512, 4096] (seed 0), Q/K/V ~ N(0, 1), block ids a
seeded random permutation of the pool.  One step = one decode token for every
sequence: pack the step on the GPU, then per layer append the new K/V and run
paged attention.  Contexts grow by one token per step.  Every layer reads a
different ~300 MB pool, larger than the 126 MB L2, so no flush is needed.

With --gpus N (torchrun, one process per GPU) each rank holds 8/N KV heads
(and the matching 32/N query heads) of a batch of 64*N sequences -- fixed
work per GPU -- and the attention outputs are all-gathered over NCCL after
every layer.

Prints one JSON line (rank 0).  --impl reference times the CPU oracle (the
reference's per-row algorithm restated) on the host cores instead.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402
import torch  # noqa: E402

# DRAM bytes (read + write) of one nf_paged_attention launch over algorithmic
# bytes, from an ncu capture (dram__bytes_read.sum + dram__bytes_write.sum) of
# the 1-layer case of the 1B workload: 317.28 MB for 307.57 MB of keys,
# values, queries, outputs and block-table entries.  Traffic scales with the
# keys read.
ATTN_TRAFFIC_RATIO = 1.0316

# resident: layers held in HBM and run per step (a full 8B step's KV, ~618 GB,
# exceeds one GPU); tok/s counts every step as `layers` layers at the measured
# per-layer time.  scaling: weak = batch grows with N (64*N sequences), strong
# = the same 256 sequences with the KV heads sharded over N GPUs.
WORKLOADS = {
    "llama3.2-1b-decode": dict(layers=16, resident=16, hq=32, hkv=8, d=64, bs=16, seqs=64, ctx_lo=512,
                               ctx_hi=4096, seed=0, scaling="weak", steps=300, cpu_sample=8,
                               metric="paged-attn decode tok/s (1B shape, 16 layers)",
                               traffic_ratio=ATTN_TRAFFIC_RATIO,
                               traffic_source="ncu capture of the 1-layer case, scaled by keys read"),
    "llama3-8b-long": dict(layers=32, resident=4, hq=32, hkv=8, d=128, bs=16, seqs=256, ctx_lo=4096,
                           ctx_hi=32768, seed=0, scaling="strong", steps=20, cpu_sample=2,
                           metric="paged-attn decode tok/s (8B shape, 32 layers, 4 resident, per-layer timed)"),
    # one continuous-batching step of the 1B shape: 4 prefill chunks of 512 tokens continuing cached
    # prefixes U[0, 2048] (rewound every step, so every timed step is this one) + 96 decodes U[256, 2048]
    "llama3.2-1b-mixed": dict(kind="mixed", layers=16, resident=16, hq=32, hkv=8, d=64, bs=16, seed=0,
                              scaling="strong", steps=30, chunks=4, chunk=512, prefix_hi=2048, decodes=96,
                              dctx_lo=256, dctx_hi=2048, seqs=100, ctx_lo=256, ctx_hi=2048, cpu_sample=8,
                              metric="mixed prefill+decode step tok/s (1B shape, 16 layers, 4x512 chunks + 96 "
                                     "decodes)"),
    # decode over shared prefixes on the 1B shape: 128 requests, each one of 4 common 1024-token
    # prefixes (64 shared blocks, imported through the prefix cache) + a unique U[64, 256] suffix
    "llama3.2-1b-prefix": dict(kind="prefix", layers=16, resident=16, hq=32, hkv=8, d=64, bs=16, seed=1,
                               scaling="strong", steps=40, seqs=128, prefixes=4, prefix_len=1024, suffix_lo=64,
                               suffix_hi=256, vocab=50257, cpu_sample=8,
                               metric="paged-attn decode tok/s over shared prefixes (1B shape, 16 layers, 128 seqs "
                                      "on 4 shared 1024-token prefixes)"),
    # the end-to-end configuration: the GPT-124M engine (fp32, context 2048, seed 0) generating 64 greedy
    # tokens for 8 requests whose prompts are U[32, 256] random ids, through Engine.add_request / step
    "gpt124m-engine": dict(kind="engine", layers=12, resident=12, hq=12, hkv=12, d=64, bs=16, seed=0,
                           scaling="weak", steps=130, requests=8, prompt_lo=32, prompt_hi=256, new_tokens=64,
                           seqs=8, ctx_lo=32, ctx_hi=320, cpu_sample=1,
                           metric="engine greedy generation tok/s (GPT-124M fp32, 8 requests x 64 new tokens)"),
}
CFG = dict(name="llama3.2-1b-decode", **WORKLOADS["llama3.2-1b-decode"])
METRIC = CFG["metric"]


def _args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--e2e-steps", type=int, default=50)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--layers", type=int, default=None, help="fewer resident layers (profiling a small case)")
    ap.add_argument("--seqs", type=int, default=None, help="fewer decode sequences (profiling a small case)")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="llama3.2-1b-decode")
    a = ap.parse_args()
    global METRIC
    CFG.clear()
    CFG.update(name=a.workload, **WORKLOADS[a.workload])
    METRIC = CFG["metric"]
    if a.steps is None:
        a.steps = CFG["steps"]
    if a.layers:  # profiling a small case: fewer resident layers (and, for the 1B shape, a shallower model)
        CFG["resident"] = a.layers
        if a.workload != "llama3-8b-long":
            CFG["layers"] = a.layers
    if a.seqs:
        CFG["seqs"] = a.seqs
    return a


def _ctx_lens(n, seed):
    if CFG.get("kind") == "prefix":
        _, group, suffix = _prefix_shape(n)
        return [CFG["prefix_len"] + len(suffix[r]) for r in range(n)]
    rng = np.random.default_rng(seed)
    return rng.integers(CFG["ctx_lo"], CFG["ctx_hi"] + 1, size=n).tolist()


def _prefix_shape(n):
    """Token ids of the shared prefixes, each request's prefix and its unique suffix (seeded)."""
    rng = np.random.default_rng(CFG["seed"])
    prefixes = [rng.integers(0, CFG["vocab"], size=CFG["prefix_len"]).tolist() for _ in range(CFG["prefixes"])]
    group = rng.integers(0, CFG["prefixes"], size=n).tolist()
    suffix = [rng.integers(0, CFG["vocab"], size=int(rng.integers(CFG["suffix_lo"], CFG["suffix_hi"] + 1))).tolist()
              for _ in range(n)]
    return prefixes, group, suffix


# ---------------------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except (OSError, FileNotFoundError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.t.join(timeout=2)
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for nm, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def _tensor_peak():
    """Dense bf16 peak for a kernel timed inside a long step: the sustained figure."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        if "bf16_tflops_sustained" in d:
            return float(d["bf16_tflops_sustained"]), "measured (sustained)"
        return float(d["bf16_tflops"]), "measured (burst)"
    return 1400.0, "fallback (sustained)"


# ---------------------------------------------------------------------------- CPU baseline (oracle)
class CpuOracleDecode:
    """The reference algorithm on the host: per-row get -> append -> cat -> matmul -> softmax -> matmul.

    One call of ``layer()`` is one layer of decode for the first ``n_sample``
    sequences of the workload (grouped-query heads restated by repeating the
    KV heads, as the reference has a single head count).  ``pos`` is held so
    every call sees the same contexts.
    """

    def __init__(self, n_sample: int | None = None, threads: int | None = None):
        from oracle.paged import OracleStore

        if threads:
            torch.set_num_threads(threads)
        n_sample = n_sample or CFG["cpu_sample"]
        self.n = n_sample
        self.ctx = _ctx_lens(CFG["seqs"], CFG["seed"])[:n_sample]
        H, D, bs = CFG["hkv"], CFG["d"], CFG["bs"]
        st = OracleStore(2, max(self.ctx) + 64, H, D, batch_size=n_sample, dtype=torch.bfloat16,
                         block_size=bs, prefix=False)
        g = torch.Generator().manual_seed(1)
        for s, c in enumerate(self.ctx):  # fill contexts block-wise (not timed)
            st.tables[s].ensure(c)
            kk = torch.randn(c, H, D, generator=g).to(torch.bfloat16)
            vv = torch.randn(c, H, D, generator=g).to(torch.bfloat16)
            for i, b in enumerate(st.tables[s].blocks):
                n = min(bs, c - i * bs)
                st.k[0][b, :n] = kk[i * bs: i * bs + n]
                st.v[0][b, :n] = vv[i * bs: i * bs + n]
            st.pos[s] = c
        self.store = st
        self.q = torch.randn(n_sample, 1, CFG["hq"] * D, generator=g).to(torch.bfloat16)
        self.k = torch.randn(n_sample, 1, H * D, generator=g).to(torch.bfloat16)

    def layer(self) -> float:
        from oracle.attention import forward_with_cache

        t0 = time.perf_counter()
        forward_with_cache(self.store, 0, self.q, self.k, self.k, CFG["hq"])  # layer 0 of 2: pos held
        return time.perf_counter() - t0

    def describe(self, calls: int, seconds: float) -> str:
        return (f"{self.n} of {CFG['seqs']} sequences (mean ctx {sum(self.ctx) / self.n:.0f}), one layer x "
                f"{calls} calls in {seconds:.1f} s, scaled to {CFG['layers']} layers")

    def rate(self, t_layer: float) -> float:
        return self.n / (CFG["layers"] * t_layer)


def cpu_decode_rate(seconds: float, threads: int | None = None):
    cpu = CpuOracleDecode(threads=threads)
    times = []
    while sum(times) < seconds:
        times.append(cpu.layer())
    t = sum(times) / len(times)
    return {"value": cpu.rate(t), "unit": "tok/s", "cores": torch.get_num_threads(),
            "sample": cpu.describe(len(times), sum(times))}


# ---------------------------------------------------------------------------- our arm
def run_ours(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    if CFG["hkv"] % world:
        raise SystemExit(f"--gpus {world} must divide {CFG['hkv']} KV heads")
    from nifre_b200.sharding import HeadShard
    shard = HeadShard(world, rank, CFG["hq"], CFG["hkv"], CFG["d"])
    hkv, hq = shard.kv_heads, shard.q_heads
    B = CFG["seqs"] * world if CFG["scaling"] == "weak" else CFG["seqs"]
    ctx = _ctx_lens(B, CFG["seed"])
    steps_total = args.warmup + args.steps + args.e2e_steps + 2
    dt = torch.bfloat16
    if CFG.get("kind") == "prefix":
        return _run_decode_timed(args, _build_prefix_cache(B, ctx, steps_total, hkv, dev, dt), B, ctx, world, rank,
                                 local, dev, dist, shard, hkv, hq)
    return _run_decode_timed(args, _build_decode_cache(B, ctx, steps_total, hkv, dev, dt, rank), B, ctx, world, rank,
                             local, dev, dist, shard, hkv, hq)


def _build_decode_cache(B, ctx, steps_total, hkv, dev, dt, rank):
    """Pool of the decode workloads: contexts filled with N(0,1) K/V over a randomly permuted free list."""
    from nifre_b200 import PagedKVCache

    L, D, bs = CFG["resident"], CFG["d"], CFG["bs"]
    max_seq = max(ctx) + steps_total + 16
    # the pool holds the contexts plus the steps' tokens (sum of ceil(ctx/bs) blocks), shuffled below
    n_blocks = sum((c + steps_total + 16 + bs - 1) // bs for c in ctx)
    cache = PagedKVCache(L, max_seq, hkv, D, device=dev, dtype=dt, block_size=bs, enable_prefix_cache=False,
                         num_blocks=n_blocks)
    cache.init_batch(B)
    g = torch.Generator().manual_seed(CFG["seed"])
    cache.block_allocator.set_free_order(torch.randperm(cache.num_blocks, generator=g).tolist())
    # fill the contexts (N(0,1) keys and values) through the append path, layer
    # by layer, in groups of sequences of at most ~1M tokens
    gd = torch.Generator(device=dev).manual_seed(CFG["seed"] + rank)
    groups, cur = [], []
    for s_ in range(B):
        if cur and sum(ctx[i] for i in cur) + ctx[s_] > (1 << 20):
            groups.append(cur)
            cur = []
        cur.append(s_)
    groups.append(cur)
    for grp in groups:
        lens = [ctx[i] for i in grp]
        plan = cache.plan(grp, lens, np.cumsum([0] + lens[:-1]).tolist())
        kfill = torch.empty(sum(lens), hkv * D, device=dev, dtype=dt)
        vfill = torch.empty_like(kfill)
        for layer in range(L):
            kfill.normal_(generator=gd)
            vfill.normal_(generator=gd)
            cache.append_step(layer, kfill, vfill, plan)
        del kfill, vfill, plan
    return cache


def _build_prefix_cache(B, ctx, steps_total, hkv, dev, dt):
    """Pool of the shared-prefix workload, built the way the engine builds it: each request imports
    the longest cached prefix (``try_load_prefix``), prefills the rest, and registers its prompt
    once complete (``register_prefix``), so later requests share the first request's prefix blocks."""
    from nifre_b200 import PagedKVCache

    L, D, bs = CFG["resident"], CFG["d"], CFG["bs"]
    prefixes, group, suffix = _prefix_shape(B)
    max_seq = max(ctx) + steps_total + 16
    n_blocks = CFG["prefixes"] * (CFG["prefix_len"] // bs) + sum(
        (len(sfx) + steps_total + 16 + bs - 1) // bs + 1 for sfx in suffix)
    cache = PagedKVCache(L, max_seq, hkv, D, device=dev, dtype=dt, block_size=bs, enable_prefix_cache=True,
                         num_blocks=n_blocks)
    cache.init_batch(B)
    gd = torch.Generator(device=dev).manual_seed(CFG["seed"])
    for r in range(B):
        tokens = prefixes[group[r]] + suffix[r]
        matched = cache.try_load_prefix(r, tokens)
        n_new = len(tokens) - matched
        plan = cache.plan([r], [n_new], [0])
        kf = torch.empty(n_new, hkv * D, device=dev, dtype=dt)
        vf = torch.empty_like(kf)
        for layer in range(L):
            kf.normal_(generator=gd)
            vf.normal_(generator=gd)
            cache.append_step(layer, kf, vf, plan)
        cache.register_prefix(r, tokens)
    cache.shared_prefix_keys = (B - len(set(group))) * CFG["prefix_len"]  # keys a cascade would not re-read
    return cache


def _run_decode_timed(args, cache, B, ctx, world, rank, local, dev, dist, shard, hkv, hq):
    from nifre_b200 import Attention

    L, L_model, D, bs = CFG["resident"], CFG["layers"], CFG["d"], CFG["bs"]
    dt = torch.bfloat16
    gd = torch.Generator(device=dev).manual_seed(CFG["seed"] + 1000 + rank)
    q_all = torch.randn(L, B, hq * D, device=dev, dtype=dt, generator=gd)
    k_all = torch.randn(L, B, hkv * D, device=dev, dtype=dt, generator=gd)
    v_all = torch.randn(L, B, hkv * D, device=dev, dtype=dt, generator=gd)
    out_loc = torch.empty(L, B, hq * D, device=dev, dtype=dt)
    gathered = torch.empty(world * B, hq * D, device=dev, dtype=dt) if world > 1 else None
    slots, ones, rows = list(range(B)), [1] * B, list(range(B))
    stream = torch.cuda.current_stream(dev)
    att_events = []

    def step(rec_layer=-1):
        p = cache.plan(slots, ones, rows, q_heads=hq)
        for layer in range(L):
            cache.append_step(layer, k_all[layer], v_all[layer], p)
            record = layer == rec_layer
            if record:
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record(stream)
            cache.attention_step(layer, q_all[layer], p, out_loc[layer])
            if record:
                e1.record(stream)
                att_events.append((e0, e1, p))
            if world > 1:
                # heads of rank r are query heads [r*hq, (r+1)*hq): (N*B, hq*D) -> (B, N*hq*D)
                shard.gather(out_loc[layer], buffer=gathered)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    cache.check_status()
    if world > 1:
        dist.barrier()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.25)
    torch.cuda.synchronize()
    e_start = torch.cuda.Event(enable_timing=True)
    e_end = torch.cuda.Event(enable_timing=True)
    e_start.record(stream)
    # the attention kernel is timed by events around one layer per step, a
    # different layer each step: events between every pair of kernels would
    # add a drain per event to the step
    for s in range(args.steps):
        step(rec_layer=s % L)
    e_end.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = e_start.elapsed_time(e_end)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    cache.check_status()
    # attention kernel: algorithmic bytes per launch / event duration
    att_ms = [a.elapsed_time(b) for a, b, _ in att_events]
    att_bytes, logical_bytes = [], []
    shared = getattr(cache, "shared_prefix_keys", 0)  # prefix keys of other sequences: read once (unique bytes)
    for _, _, p in att_events:
        kv = int(p.kv_lens.sum())
        nblk = int(((p.kv_lens + bs - 1) // bs).sum())
        att_bytes.append((kv - shared) * hkv * D * 2 * 2 + 2 * B * hq * D * 2 + 4 * nblk + 16 * B)
        logical_bytes.append(kv * hkv * D * 2 * 2 + 2 * B * hq * D * 2 + 4 * nblk + 16 * B)
    from nifre_b200 import _lib
    att_path = _lib.load().nf_last_attention_path()
    att_avg_ms = sum(att_ms) / len(att_ms)
    achieved = (sum(att_bytes) / len(att_bytes)) / (att_avg_ms * 1e-3) / 1e9
    peak, peak_kind = _peaks()

    # e2e through the public drop-in API with host buffers
    e2e = None
    if args.e2e_steps > 0:
        attn = Attention(hq, D)
        hq_host = torch.empty(L, B, 1, hq * D, dtype=dt).pin_memory()
        hk_host = torch.empty(L, B, 1, hkv * D, dtype=dt).pin_memory()
        hv_host = torch.empty_like(hk_host).pin_memory()
        ho_host = torch.empty(L, B, 1, hq * D, dtype=dt).pin_memory()
        hq_host.copy_(q_all.view(L, B, 1, -1).cpu())
        hk_host.copy_(k_all.view(L, B, 1, -1).cpu())
        hv_host.copy_(v_all.view(L, B, 1, -1).cpu())

        def e2e_step():
            # the step's inputs go up in one copy per tensor, its outputs come
            # down in one copy: each layer runs through Attention.forward
            qd_all = hq_host.to(dev, non_blocking=True)
            kd_all = hk_host.to(dev, non_blocking=True)
            vd_all = hv_host.to(dev, non_blocking=True)
            outs = []
            for layer in range(L):
                o = attn(qd_all[layer], kd_all[layer], vd_all[layer], kv_cache=cache, layer_id=layer,
                         cache_batch_indices=slots)
                if world > 1:
                    o = shard.gather(o.view(B, -1), buffer=gathered).view(B, 1, world * hq * D)[:, :, : hq * D]
                outs.append(o)
            ho_host.copy_(torch.stack(outs), non_blocking=True)

        e2e_step()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(args.e2e_steps - 1):
            e2e_step()
        b.record(stream)
        torch.cuda.synchronize()
        ems = a.elapsed_time(b)
        if world > 1:
            t = torch.tensor([ems], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ems = float(t.item())
        cache.check_status()
        n_e2e = args.e2e_steps - 1
        e2e = {"value": B * n_e2e / (ems * 1e-3) * L / L_model, "unit": "tok/s",
               "h2d_bytes_per_step": L * B * (hq + 2 * hkv) * D * 2,
               "d2h_bytes_per_step": L * B * hq * D * 2,
               "ms_per_step": ems / n_e2e,
               "path": "nifre_b200.Attention.forward per layer; the step's q/k/v copied up from pinned host memory "
                       "in one copy per tensor, its outputs copied down in one"}

    if rank == 0:
        cpu = None
        if not args.no_cpu_baseline:
            cpu = cpu_decode_rate(12.0)
            cpu["kind"] = "port"
        line = {
            "metric": METRIC, "value": B * args.steps / (ms * 1e-3) * L / L_model, "unit": "tok/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms / args.steps * L_model / L,
            "higher_is_better": True, "scaling": CFG["scaling"], "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) Q/K/V, random block permutation)",
            "config": {"workload": CFG["name"], "layers": L_model, "layers_timed": L, "q_heads": CFG["hq"],
                       "kv_heads": CFG["hkv"], "head_dim": D, "block_size": bs,
                       "seqs_per_gpu_x_heads": f"{B} seqs x {hkv} kv heads",
                       "global_batch": B,
                       "ctx": (f"U[{CFG['ctx_lo']},{CFG['ctx_hi']}] + step" if "ctx_lo" in CFG else
                               f"{CFG['prefix_len']}-token prefix (one of {CFG['prefixes']}, shared blocks) + "
                               f"U[{CFG['suffix_lo']},{CFG['suffix_hi']}] suffix + step"),
                       "parallelism": f"kv-head shard x{world}" if world > 1 else "single GPU",
                       "method": ("all layers run every step" if L == L_model else
                                  f"{L} resident layers run per step; tok/s and ms_per_step scaled to "
                                  f"{L_model} layers at the measured per-layer time"),
                       "l2": ("inputs larger than L2 (each layer reads a distinct pool of >=300 MB)"
                              if not shared else
                              "each layer reads a distinct pool; shared prefix blocks (16 MB per layer) are read by "
                              "every sequence that imported them: the roofline counts them once (unique bytes)")},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak,
                         "traffic": (CFG["traffic_ratio"] * sum(att_bytes) / len(att_bytes)
                                     if CFG.get("traffic_ratio") else None),
                         "traffic_source": CFG.get("traffic_source"),
                         "kernel": "nf_paged_attention",
                         "kernel_path": {0: "per-warp cp.async", 1: "tensor map, one copy per block",
                                         2: "tensor map, one copy per head"}.get(att_path, str(att_path)),
                         "peak_source": peak_kind, "avg_launch_us": att_avg_ms * 1e3,
                         **({"bytes": "unique (shared prefix blocks once)",
                             "achieved_logical": (sum(logical_bytes) / len(logical_bytes)) / (att_avg_ms * 1e-3) / 1e9}
                            if shared else {})},
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": args.steps * (1 + 2 * L),
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    if CFG.get("kind") == "engine":
        cpu = cpu_engine_rate(max(5.0, 1.0 * args.steps / 10), threads=threads)
        line = {"impl": "reference", "metric": METRIC, "value": cpu["value"], "unit": "tok/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": CFG["scaling"],
                "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
                "config": {"workload": CFG["name"], "model": "GPT-124M (12 layers, 12 heads, d 64, context 2048)"},
                "cpu_baseline": dict(cpu, kind="port"),
                "e2e": {"value": cpu["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return
    if CFG.get("kind") == "mixed":
        cpu = CpuOracleMixed(threads=threads)
        for _ in range(args.warmup):
            cpu.layer()
        pairs = [cpu.layer() for _ in range(args.steps)]
        v = cpu.rate(sum(a for a, _ in pairs) / len(pairs), sum(b for _, b in pairs) / len(pairs))
        times = [a + b for a, b in pairs]
    else:
        cpu = CpuOracleDecode(threads=threads)
        for _ in range(args.warmup):
            cpu.layer()
        times = [cpu.layer() for _ in range(args.steps)]
        v = cpu.rate(sum(times) / len(times))
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": CFG["scaling"],
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": CFG["name"], "layers": CFG["layers"], "q_heads": CFG["hq"],
                       "kv_heads": CFG["hkv"], "head_dim": CFG["d"], "block_size": CFG["bs"]},
            "cpu_baseline": {"value": v, "unit": "tok/s", "cores": torch.get_num_threads(), "kind": "port",
                             "sample": cpu.describe(len(times), sum(times)) + "; each step = one such call"},
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------- mixed step (prefill + decode)
def _mixed_shape():
    rng = np.random.default_rng(CFG["seed"])
    prefix = rng.integers(0, CFG["prefix_hi"] + 1, size=CFG["chunks"]).tolist()
    dctx = rng.integers(CFG["dctx_lo"], CFG["dctx_hi"] + 1, size=CFG["decodes"]).tolist()
    return prefix, dctx


def _mixed_flops(prefix, hq, d, chunk):
    """Algorithmic prefill FLOPs of one layer: unmasked causal pairs only, 4*Hq*D per pair."""
    return 4.0 * hq * d * sum(chunk * p + chunk * (chunk + 1) / 2 for p in prefix)


class CpuOracleMixed:
    """The reference algorithm on the host for the mixed step: one 512-token chunk and 8 decodes per call."""

    def __init__(self, threads: int | None = None):
        from oracle.paged import OracleStore

        if threads:
            torch.set_num_threads(threads)
        prefix, dctx = _mixed_shape()
        self.prefix, self.dctx = prefix, dctx
        H, D, bs, C = CFG["hkv"], CFG["d"], CFG["bs"], CFG["chunk"]
        self.nd = min(CFG["cpu_sample"], len(dctx))
        ctx = [prefix[0]] + dctx[: self.nd]
        st = OracleStore(2, max(ctx) + C + 64, H, D, batch_size=len(ctx), dtype=torch.bfloat16, block_size=bs,
                         prefix=False)
        g = torch.Generator().manual_seed(1)
        for sl, c in enumerate(ctx):
            if c == 0:
                continue
            st.tables[sl].ensure(c)
            kk = torch.randn(c, H, D, generator=g).to(torch.bfloat16)
            vv = torch.randn(c, H, D, generator=g).to(torch.bfloat16)
            for i, b in enumerate(st.tables[sl].blocks):
                n = min(bs, c - i * bs)
                st.k[0][b, :n] = kk[i * bs: i * bs + n]
                st.v[0][b, :n] = vv[i * bs: i * bs + n]
            st.pos[sl] = c
        self.store = st
        hq = CFG["hq"]
        self.qc = torch.randn(1, C, hq * D, generator=g).to(torch.bfloat16)
        self.kc = torch.randn(1, C, H * D, generator=g).to(torch.bfloat16)
        self.qd = torch.randn(self.nd, 1, hq * D, generator=g).to(torch.bfloat16)
        self.kd = torch.randn(self.nd, 1, H * D, generator=g).to(torch.bfloat16)

    def layer(self) -> tuple[float, float]:
        from oracle.attention import forward_with_cache

        t0 = time.perf_counter()
        forward_with_cache(self.store, 0, self.qc, self.kc, self.kc, CFG["hq"], slots=[0])
        t1 = time.perf_counter()
        forward_with_cache(self.store, 0, self.qd, self.kd, self.kd, CFG["hq"], slots=list(range(1, self.nd + 1)))
        return t1 - t0, time.perf_counter() - t1

    def rate(self, t_chunk: float, t_dec: float) -> float:
        t_layer = len(self.prefix) * t_chunk + len(self.dctx) / self.nd * t_dec
        tokens = len(self.prefix) * CFG["chunk"] + len(self.dctx)
        return tokens / (CFG["layers"] * t_layer)

    def describe(self, calls: int, seconds: float) -> str:
        return (f"one 512-token chunk (prefix {self.prefix[0]}) and {self.nd} of {len(self.dctx)} decodes, one "
                f"layer x {calls} calls in {seconds:.1f} s, scaled to 4 chunks + 96 decodes x {CFG['layers']} layers")


def cpu_mixed_rate(seconds: float, threads: int | None = None):
    cpu = CpuOracleMixed(threads=threads)
    tc, td = [], []
    while sum(tc) + sum(td) < seconds:
        a, b = cpu.layer()
        tc.append(a)
        td.append(b)
    return {"value": cpu.rate(sum(tc) / len(tc), sum(td) / len(td)), "unit": "tok/s",
            "cores": torch.get_num_threads(), "sample": cpu.describe(len(tc), sum(tc) + sum(td))}


def run_mixed(args):
    from nifre_b200 import PagedKVCache
    from nifre_b200.sharding import HeadShard

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    shard = HeadShard(world, rank, CFG["hq"], CFG["hkv"], CFG["d"])
    hkv, hq = shard.kv_heads, shard.q_heads
    L, D, bs, C = CFG["layers"], CFG["d"], CFG["bs"], CFG["chunk"]
    prefix, dctx = _mixed_shape()
    P, ND = len(prefix), len(dctx)
    B = P + ND
    steps_total = args.warmup + args.steps + args.e2e_steps + 2
    max_seq = max(max(prefix) + C, max(dctx) + steps_total) + 16
    n_blocks = sum((p + C + bs - 1) // bs for p in prefix) + sum((c + steps_total + 16 + bs - 1) // bs for c in dctx)
    dt = torch.bfloat16
    cache = PagedKVCache(L, max_seq, hkv, D, device=dev, dtype=dt, block_size=bs, enable_prefix_cache=False,
                         num_blocks=n_blocks)
    cache.init_batch(B)
    g = torch.Generator().manual_seed(CFG["seed"])
    cache.block_allocator.set_free_order(torch.randperm(cache.num_blocks, generator=g).tolist())
    gd = torch.Generator(device=dev).manual_seed(CFG["seed"] + rank)
    ctx = prefix + dctx
    fill = [i for i in range(B) if ctx[i] > 0]
    lens = [ctx[i] for i in fill]
    plan = cache.plan(fill, lens, np.cumsum([0] + lens[:-1]).tolist())
    kfill = torch.empty(sum(lens), hkv * D, device=dev, dtype=dt)
    vfill = torch.empty_like(kfill)
    for layer in range(L):
        kfill.normal_(generator=gd)
        vfill.normal_(generator=gd)
        cache.append_step(layer, kfill, vfill, plan)
    del kfill, vfill, plan
    q_lens = [C] * P + [1] * ND
    starts = np.cumsum([0] + q_lens[:-1]).tolist()
    T = sum(q_lens)
    q_all = torch.randn(L, T, hq * D, device=dev, dtype=dt, generator=gd)
    k_all = torch.randn(L, T, hkv * D, device=dev, dtype=dt, generator=gd)
    v_all = torch.randn(L, T, hkv * D, device=dev, dtype=dt, generator=gd)
    out_loc = torch.empty(L, T, hq * D, device=dev, dtype=dt)
    gathered = torch.empty(world * T, hq * D, device=dev, dtype=dt) if world > 1 else None
    slots = list(range(B))
    stream = torch.cuda.current_stream(dev)
    kev = []

    def rewind():  # every step continues the same prefixes (the decodes keep growing)
        for i in range(P):
            cache._set_pos(i, prefix[i])

    def step(rec_layer=-1, host=None):
        rewind()
        p = cache.plan(slots, q_lens, starts, q_heads=hq)
        if host is not None:  # the step's inputs up in one copy per tensor
            qa, ka, va = (host[i].to(dev, non_blocking=True) for i in range(3))
        for layer in range(L):
            if host is not None:
                qd, kd, vd = qa[layer], ka[layer], va[layer]
            else:
                qd, kd, vd = q_all[layer], k_all[layer], v_all[layer]
            cache.append_step(layer, kd, vd, p)
            ev = None
            if layer == rec_layer:
                ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
                kev.append((ev, p))
            cache.attention_step(layer, qd, p, out_loc[layer], events=ev)
            o = out_loc[layer]
            if world > 1:
                o = shard.gather(o, buffer=gathered)
                if host is not None:
                    host[3][layer].copy_(o[:, : hq * D], non_blocking=True)
        if host is not None and world == 1:  # the step's outputs down in one copy
            host[3].copy_(out_loc, non_blocking=True)
        return p

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    cache.check_status()
    if world > 1:
        dist.barrier()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.25)
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    # the kernels are timed by events around one layer per step, a different
    # layer each step (events between every pair of kernels would add a
    # drain per event to the step, and keep the decode from starting beside
    # the KV append)
    for s in range(args.steps):
        step(rec_layer=s % L)
    e1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    cache.check_status()
    pre_ms = [a[0].elapsed_time(a[1]) for a, _ in kev]
    dec_ms = [a[1].elapsed_time(a[2]) for a, _ in kev]
    pre_avg, dec_avg = sum(pre_ms) / len(pre_ms), sum(dec_ms) / len(dec_ms)
    flops = _mixed_flops(prefix, hq, D, C)  # this rank's heads
    dec_bytes = []
    for _, p in kev:
        kv = p.kv_lens[P:]
        dec_bytes.append(int(kv.sum()) * hkv * D * 4 + 2 * ND * hq * D * 2 + 4 * int(((kv + bs - 1) // bs).sum()))
    hbm_peak, hbm_kind = _peaks()
    tf_peak, tf_kind = _tensor_peak()
    # e2e: the same steps through the cache API with q/k/v copied from pinned host memory and the
    # attention output copied back every layer
    e2e = None
    if args.e2e_steps > 1:
        host = (q_all.cpu().pin_memory(), k_all.cpu().pin_memory(), v_all.cpu().pin_memory(),
                torch.empty(L, T, hq * D * world, dtype=dt).pin_memory())
        step(host=host)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(args.e2e_steps - 1):
            step(host=host)
        b.record(stream)
        torch.cuda.synchronize()
        ems = a.elapsed_time(b)
        if world > 1:
            t = torch.tensor([ems], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ems = float(t.item())
        n = args.e2e_steps - 1
        e2e = {"value": T * n / (ems * 1e-3), "unit": "tok/s",
               "h2d_bytes_per_step": L * T * (hq + 2 * hkv) * D * 2, "d2h_bytes_per_step": L * T * hq * world * D * 2,
               "ms_per_step": ems / n,
               "path": "PagedKVCache.plan/append_step/attention_step; the step's q/k/v up from pinned host memory in "
                       "one copy per tensor, outputs down in one"}
        cache.check_status()
    if rank == 0:
        cpu = None
        if not args.no_cpu_baseline:
            cpu = cpu_mixed_rate(12.0)
            cpu["kind"] = "port"
        pre_tf = flops * world / (pre_avg * 1e-3) / 1e12
        dec_gbs = (sum(dec_bytes) / len(dec_bytes)) / (dec_avg * 1e-3) / 1e9
        line = {
            "metric": METRIC, "value": T * args.steps / (ms * 1e-3), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": CFG["scaling"], "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) Q/K/V, random block permutation)",
            "config": {"workload": CFG["name"], "layers": L, "q_heads": CFG["hq"], "kv_heads": CFG["hkv"],
                       "head_dim": D, "block_size": bs, "prefill_chunks": P, "chunk_tokens": C,
                       "prefixes": prefix, "decodes": ND, "decode_ctx": f"U[{CFG['dctx_lo']},{CFG['dctx_hi']}]",
                       "tokens_per_step": T, "global_batch": B,
                       "parallelism": f"kv-head shard x{world}" if world > 1 else "single GPU",
                       "method": "prefill slots rewound to their prefixes every step; decodes grow by one",
                       "l2": "inputs larger than L2 (each layer reads a distinct pool of ~250 MB)"},
            "roofline": {"bound": "tensor", "achieved": pre_tf, "peak": tf_peak, "unit": "TFLOP/s",
                         "frac": pre_tf / tf_peak, "traffic": None, "kernel": "nf_prefill_attention",
                         "peak_source": tf_kind, "avg_launch_us": pre_avg * 1e3,
                         "flops_per_launch": flops * world,
                         "flops_counted": "4*Hq*D per unmasked (query, key) pair"},
            "roofline_decode": {"bound": "hbm", "achieved": dec_gbs, "peak": hbm_peak, "unit": "GB/s",
                                "frac": dec_gbs / hbm_peak, "kernel": "nf_paged_attention",
                                "peak_source": hbm_kind, "avg_launch_us": dec_avg * 1e3},
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": args.steps * (1 + 3 * L),
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# ---------------------------------------------------------------------------- end-to-end engine (GPT-124M)
def _engine_prompts(seed):
    """The workload's prompts: Python's random seeded with ``seed`` (seed 0 is the end-to-end configuration)."""
    import random
    rnd = random.Random(seed)
    out = []
    for _ in range(CFG["requests"]):
        n = rnd.randint(CFG["prompt_lo"], CFG["prompt_hi"])
        out.append([rnd.randrange(50257) for _ in range(n)])
    return out


def _engine_model(dev):
    from nifre_b200.gpt import GPT_CONFIG_124M, GptModel
    cfg = dict(GPT_CONFIG_124M, context_length=2048)
    torch.manual_seed(CFG["seed"])
    return GptModel(cfg).eval().to(dev)


def cpu_engine_rate(seconds: float, threads: int | None = None):
    """The reference's greedy generation on the host cores (oracle/engine.py port, one request at a time as the
    reference's rows are): decode tok/s over the first prompts of the workload, stopped after ``seconds``."""
    from oracle.engine import greedy_generate
    if threads:
        torch.set_num_threads(threads)
    model = _engine_model("cpu")
    toks, spent, n_req = 0, 0.0, 0
    for prompt in _engine_prompts(CFG["seed"]):
        _, t, n = greedy_generate(model, prompt, CFG["new_tokens"])
        toks += n
        spent += t
        n_req += 1
        if spent >= seconds:
            break
    return {"value": toks / spent, "unit": "tok/s", "cores": torch.get_num_threads(),
            "sample": f"{n_req} of {CFG['requests']} requests, {toks} decode steps of one request each "
                      f"({spent:.1f} s), prefill excluded"}


def run_engine(args):
    """Greedy generation through the engine: every timed step is one Engine.step() (host scheduling, one
    upload of the step's ids/positions, the flat forward, one download of the sampled tokens); N GPUs run N
    independent replicas."""
    from nifre_b200 import Engine, GptInferenceModel
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    torch.backends.cuda.matmul.allow_tf32 = False  # fp32 GEMMs, as the parity test runs them
    eng = Engine(GptInferenceModel(_engine_model(dev)), max_concurrent_requests=CFG["requests"], device=dev,
                 prefill_chunk_size=128, max_tokens_per_step=2048)
    stream = torch.cuda.current_stream(dev)
    stats = {"steps": 0, "tokens": 0, "h2d": 0, "d2h": 0, "launches": 0, "rec": [], "record": False}

    def generation(seed):
        ids = [eng.add_request(p, CFG["new_tokens"]) for p in _engine_prompts(seed)]
        while eng.step():
            stats["steps"] += 1
        done = eng.get_completed()
        stats["tokens"] += sum(len(done[i].output_token_ids) for i in ids)

    generation(1000 + rank)  # warm-up generation: builds the cache, the workspaces and cuBLAS handles
    for w in range(args.warmup - 1):
        generation(2000 + w)
    cache = eng.cache
    plan_fn, append_fn, attn_fn = cache.plan, cache.append_step, cache.attention_step
    run_fn = eng.model_runner.run_step
    last = {}

    def plan_w(*a, **k):
        p = plan_fn(*a, **k)
        last["plan"] = p
        stats["h2d"] += p.upload_bytes + 16 * p.n_tokens  # step metadata, token ids and positions (int64)
        stats["launches"] += 1
        return p

    def append_w(layer, *a, **k):
        stats["launches"] += 1
        return append_fn(layer, *a, **k)

    def attn_w(layer, q, p, out, *a, **k):
        stats["launches"] += (p.n_tiles > 0) + (p.n_casc_tasks > 0) + (p.decode_units > 0)
        if stats["record"] and layer == stats["steps"] % cache.num_layers and p.n_tiles == 0 \
                and (p.q_lens == 1).all():
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
            stats["rec"].append((ev, p))
            return attn_fn(layer, q, p, out, *a, events=ev, **k)
        return attn_fn(layer, q, p, out, *a, **k)

    def run_w(*a, **k):
        replays = eng.model_runner.graph_replays
        pre, dec = run_fn(*a, **k)
        if eng.model_runner.graph_replays != replays:  # a replayed step: its layers' kernels ran from the graph
            p = last["plan"]
            stats["launches"] += cache.num_layers * (1 + (p.n_casc_tasks > 0) + (p.decode_units > 0))
        n = sum(t is not None for t in pre) + len(dec)
        stats["h2d"] += 8 * n  # sampled rows
        stats["d2h"] += 8 * n  # sampled tokens
        return pre, dec

    cache.plan, cache.append_step, cache.attention_step, eng.model_runner.run_step = plan_w, append_w, attn_w, run_w
    for k in ("steps", "tokens", "h2d", "d2h", "launches"):
        stats[k] = 0
    if world > 1:
        dist.barrier()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.25)
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    gen = 0
    while stats["steps"] < args.steps:
        generation(gen)  # seed 0 first: the end-to-end configuration's prompts
        gen += 1
    e1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1)
    tokens, steps, launches, h2d, d2h = (stats[k] for k in ("tokens", "steps", "launches", "h2d", "d2h"))
    replays = eng.model_runner.graph_replays
    # the attention kernel's duration: events around one layer per decode step of an untimed generation
    # run eagerly (graph replays run the same kernels but cannot be split by events)
    eng.model_runner.use_cuda_graphs, stats["record"] = False, True
    generation(3000 + rank)
    torch.cuda.synchronize()
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        n = torch.tensor([tokens], device=dev, dtype=torch.float64)
        dist.all_reduce(n)
        tokens = int(n.item())
    cache.check_status()
    att_ms = [a[1].elapsed_time(a[2]) for a, _ in stats["rec"]]
    att_bytes = [int(p.kv_lens.sum()) * CFG["hkv"] * CFG["d"] * 4 * 2 + 2 * p.n_tokens * CFG["hq"] * CFG["d"] * 4
                 for _, p in stats["rec"]]
    hbm_peak, hbm_kind = _peaks()
    if rank == 0:
        cpu = None
        if not args.no_cpu_baseline:
            cpu = cpu_engine_rate(12.0)
            cpu["kind"] = "port"
        att_avg = sum(att_ms) / max(1, len(att_ms))
        gbs = (sum(att_bytes) / max(1, len(att_bytes))) / (att_avg * 1e-3) / 1e9 if att_ms else None
        value = tokens / (ms * 1e-3)
        line = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": steps,
            "warmup": args.warmup, "ms_per_step": ms / steps, "higher_is_better": True, "scaling": CFG["scaling"],
            "vs_baseline": None, "dtype": "fp32", "data": "synthetic (random-init GPT-124M, seed 0; prompts of "
                                                           "U[32, 256] random ids, seeded)",
            "config": {"workload": CFG["name"], "model": "GPT-124M (12 layers, 12 heads, d 64, context 2048)",
                       "global_batch": CFG["requests"] * world, "new_tokens": CFG["new_tokens"],
                       "engine": "Engine(max_concurrent_requests=8, prefill_chunk_size=128, "
                                 "max_tokens_per_step=2048)", "generations": gen,
                       "decode_steps_replayed_from_cuda_graph": replays,
                       "parallelism": f"{world} independent replicas" if world > 1 else "single GPU",
                       "l2": "not flushed: the per-step working set (weights 0.5 GB) exceeds L2"},
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm_peak, "unit": "GB/s",
                         "frac": gbs / hbm_peak if gbs else None, "traffic": None, "kernel": "nf_paged_attention",
                         "peak_source": hbm_kind, "avg_launch_us": att_avg * 1e3,
                         "note": "decode steps of 8 rows: a few MB per launch, latency-bound; the step is "
                                 "dominated by the fp32 projections (cuBLAS); timed in an untimed eager "
                                 "generation after the timed region"},
            "cpu_baseline": cpu,
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": h2d / steps,
                    "d2h_bytes_per_step": d2h / steps,
                    "path": "Engine.add_request/step/get_completed: prompts and tokens on the host; every step "
                            "uploads its metadata, ids, positions and sampled rows and downloads the sampled "
                            "tokens (value is this end-to-end rate)"},
            "gpu_launches": launches, "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    args = _args()
    mixed = CFG.get("kind") == "mixed"
    if args.impl == "reference":
        run_reference(args)
    elif mixed:
        run_mixed(args)
    elif CFG.get("kind") == "engine":
        run_engine(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
