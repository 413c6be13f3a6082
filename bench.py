#!/usr/bin/env python
"""Benchmark of the ragged paged-attention path on B200.

Headline workload (default): Llama-3.2-1B-shaped paged decode, bfloat16 -- 16
layers, 32 query heads, 8 KV heads, head_dim 64, block size 16, 64 sequences
with context lengths uniform in [512, 4096] (seed 0), Q/K/V ~ N(0, 1), block
ids a seeded random permutation of the pool.  One step = one decode token for
every sequence: pack the step on the GPU, then per layer append the new K/V
and run paged attention.  Contexts grow by one token per step.  Every layer
reads a different ~300 MB pool, larger than the 126 MB L2, so no flush is
needed.

The same JSON line carries two sub-results measured in the same run, each
with its own kernel roofline: the Llama-3-8B-shaped long-context decode (256
sequences, contexts U[4096, 32768], head_dim 128; HBM roofline of the decode
kernel) and the mixed continuous-batching step (4 prefill chunks of 512
tokens over cached prefixes plus 96 decodes; tensor roofline of the prefill
kernel, HBM roofline of the decode kernel).

With --gpus N (torchrun, one process per GPU) each rank holds 8/N KV heads
(and the matching 32/N query heads); the 1B decode keeps the work per GPU
fixed (64*N sequences), the 8B decode and the mixed step shard one batch, and
every layer's attention kernels store their output rows into all ranks'
gathered buffers over NVLink (peer stores through CUDA IPC mappings) and end
once every rank's rows are in place: no collective library call per layer.

Prints one JSON line (rank 0).  --impl reference times the reference's own
CPU attention path (installed unmodified in baseline/_ref, grouped-query heads
stored expanded to the query head count) on the host cores instead, or the
CPU port of it when that install is absent.
"""

from __future__ import annotations

import argparse
import contextlib
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
# = the same batch with the KV heads sharded over N GPUs.
WORKLOADS = {
    "llama3.2-1b-decode": dict(layers=16, resident=16, hq=32, hkv=8, d=64, bs=16, seqs=64, ctx_lo=512,
                               ctx_hi=4096, seed=0, scaling="weak", steps=300, cpu_sample=8,
                               metric="paged-attn decode tok/s (1B shape, 16 layers)",
                               traffic_ratio=ATTN_TRAFFIC_RATIO,
                               traffic_source="ncu capture of the 1-layer case, scaled by keys read"),
    "llama3-8b-long": dict(layers=32, resident=4, hq=32, hkv=8, d=128, bs=16, seqs=256, ctx_lo=4096,
                           ctx_hi=32768, seed=0, scaling="strong", steps=20, cpu_sample=2,
                           metric="paged-attn decode tok/s (8B shape, 32 layers, per-layer timed)"),
    # one continuous-batching step of the 1B shape: 4 prefill chunks of 512 tokens continuing cached
    # prefixes U[0, 2048] (rewound every step, so every timed step is this one) + 96 decodes U[256, 2048]
    "llama3.2-1b-mixed": dict(kind="mixed", layers=16, resident=16, hq=32, hkv=8, d=64, bs=16, seed=0,
                              scaling="strong", steps=30, chunks=4, chunk=512, prefix_hi=2048, decodes=96,
                              dctx_lo=256, dctx_hi=2048, seqs=100, ctx_lo=256, ctx_hi=2048, cpu_sample=8,
                              metric="mixed prefill+decode step tok/s (1B shape, 16 layers, 4x512 chunks + 96 "
                                     "decodes)"),
    # the 1B decode step's input projection fused with the KV append: 64 rows x d_model 2048 against the stacked
    # q/k/v weights (3072 x 2048, bf16, a distinct weight per layer), k/v scattered into the paged pools
    "llama3.2-1b-qkv": dict(kind="qkv", layers=16, resident=16, hq=32, hkv=8, d=64, bs=16, seqs=64, ctx_lo=512,
                            ctx_hi=4096, seed=0, scaling="weak", steps=50, d_model=2048, cpu_sample=8,
                            metric="fused qkv projection + kv append, rows/s (1B shape, 64 decode rows, 16 layers)"),
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

# sub-results of the default run: (workload, resident layers, timed steps)
SUB_RESULTS = (("llama3-8b-long", 1, 12), ("llama3.2-1b-mixed", 16, 16), ("llama3.2-1b-prefix", 16, 20),
               ("llama3.2-1b-qkv", 16, 30), ("gpt124m-engine", 12, 130))


def _args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--e2e-steps", type=int, default=50)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sub", action="store_true", help="skip the 8B-decode and mixed-step sub-results")
    ap.add_argument("--layers", type=int, default=None, help="fewer resident layers (profiling a small case)")
    ap.add_argument("--seqs", type=int, default=None, help="fewer decode sequences (profiling a small case)")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="llama3.2-1b-decode")
    a = ap.parse_args()
    _use_workload(a.workload)
    if a.steps is None:
        a.steps = CFG["steps"]
    if a.layers:  # profiling a small case: fewer resident layers (and, for the 1B shape, a shallower model)
        CFG["resident"] = a.layers
        if a.workload != "llama3-8b-long":
            CFG["layers"] = a.layers
    if a.seqs:
        CFG["seqs"] = a.seqs
    return a


def _use_workload(name: str, **over) -> None:
    global METRIC
    CFG.clear()
    CFG.update(name=name, **WORKLOADS[name])
    CFG.update(over)
    METRIC = CFG["metric"]


@contextlib.contextmanager
def _workload(name: str, **over):
    """Switch the workload for a sub-result; the headline's is restored after."""
    saved = dict(CFG)
    _use_workload(name, **over)
    try:
        yield
    finally:
        global METRIC
        CFG.clear()
        CFG.update(saved)
        METRIC = CFG["metric"]


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


def _mixed_shape():
    rng = np.random.default_rng(CFG["seed"])
    prefix = rng.integers(0, CFG["prefix_hi"] + 1, size=CFG["chunks"]).tolist()
    dctx = rng.integers(CFG["dctx_lo"], CFG["dctx_hi"] + 1, size=CFG["decodes"]).tolist()
    return prefix, dctx


def _mixed_flops(prefix, hq, d, chunk):
    """Algorithmic prefill FLOPs of one layer: unmasked causal pairs only, 4*Hq*D per pair."""
    return 4.0 * hq * d * sum(chunk * p + chunk * (chunk + 1) / 2 for p in prefix)


def _stratified(values, n):
    """Indices of n of the values at evenly spaced quantiles, so that the sample's mean matches the population's."""
    values = np.asarray(values)
    n = min(n, len(values))
    order = np.argsort(values, kind="stable")
    at = ((np.arange(n) + 0.5) * len(values) / n).astype(np.int64)
    return sorted(order[at].tolist())


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


def _tensor_peaks():
    """Dense bf16 peaks: (burst, sustained, source).  The burst figure is the one for a kernel timed
    alone or inside a short timed region (milliseconds); the sustained one holds under the power cap in
    regions of seconds."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        burst = float(d["bf16_tflops"])
        return burst, float(d.get("bf16_tflops_sustained", burst)), "measured"
    return 1590.0, 1400.0, "fallback"


# ---------------------------------------------------------------------------- CPU baselines
# Two CPU forms of the path, timed on the host cores of the GPU box in the same run:
#  * "reference": the reference's own Attention._forward_with_cache over its own PagedKVCache
#    (src/inference/attention.py:77-152, paged_kv_cache.py:107-142), installed unmodified into
#    baseline/_ref by baseline/install_ref.sh.  The reference has one head count for queries and keys,
#    so the grouped-query shapes run with the KV heads stored repeated to the query head count
#    ("MHA-expanded"): the same outputs, 4x the KV bytes of the 8-KV-head model.
#  * "port": the oracle's restatement of that algorithm (oracle/attention.py, oracle/paged.py), which
#    keeps the 8 KV heads and expands them only for the matmuls.
# Each times one layer of a bounded sample of the workload's sequences, chosen at evenly spaced
# quantiles of the context lengths so that the sample's mean context matches the batch's.

def _reference_modules():
    """(Attention, PagedKVCache) of the reference installed in baseline/_ref, or None."""
    ref = ROOT / "baseline" / "_ref"
    if not (ref / "inference" / "attention.py").exists():
        return None
    if str(ref) not in sys.path:
        sys.path.insert(0, str(ref))
    try:
        from inference.attention import Attention
        from inference.paged_kv_cache import PagedKVCache
    except Exception:  # noqa: BLE001 -- an unusable install is reported as absent
        return None
    return Attention, PagedKVCache


class _CpuDecodeBase:
    """A bounded sample of the decode workload's sequences on the host: subclasses fill the store."""

    kind = ""

    def __init__(self, n_sample: int | None = None, threads: int | None = None):
        if threads:
            torch.set_num_threads(threads)
        n_sample = n_sample or CFG["cpu_sample"]
        population = _ctx_lens(CFG["seqs"], CFG["seed"])
        self.pop_mean = float(np.mean(population))
        self.ctx = [population[i] for i in _stratified(population, n_sample)]
        self.n = len(self.ctx)
        self.g = torch.Generator().manual_seed(1)

    def describe(self, calls: int, seconds: float) -> str:
        return (f"{self.n} of {CFG['seqs']} sequences at evenly spaced context quantiles (mean ctx "
                f"{sum(self.ctx) / self.n:.0f}, batch mean {self.pop_mean:.0f}), one layer x {calls} calls in "
                f"{seconds:.1f} s, scaled to {CFG['layers']} layers")

    def rate(self, t_layer: float) -> float:
        return self.n / (CFG["layers"] * t_layer)


class CpuOracleDecode(_CpuDecodeBase):
    """The oracle port: per-row get -> append -> cat -> matmul -> softmax -> matmul, KV heads kept at Hkv.

    ``pos`` is held (layer 0 of a 2-layer store), so every call sees the same contexts.
    """

    kind = "port"

    def __init__(self, n_sample: int | None = None, threads: int | None = None):
        from oracle.paged import OracleStore

        super().__init__(n_sample, threads)
        H, D, bs = CFG["hkv"], CFG["d"], CFG["bs"]
        st = OracleStore(2, max(self.ctx) + 64, H, D, batch_size=self.n, dtype=torch.bfloat16, block_size=bs,
                         prefix=False)
        for s, c in enumerate(self.ctx):  # fill contexts block-wise (not timed)
            st.tables[s].ensure(c)
            kk = torch.randn(c, H, D, generator=self.g).to(torch.bfloat16)
            vv = torch.randn(c, H, D, generator=self.g).to(torch.bfloat16)
            for i, b in enumerate(st.tables[s].blocks):
                n = min(bs, c - i * bs)
                st.k[0][b, :n] = kk[i * bs: i * bs + n]
                st.v[0][b, :n] = vv[i * bs: i * bs + n]
            st.pos[s] = c
        self.store = st
        self.q = torch.randn(self.n, 1, CFG["hq"] * D, generator=self.g).to(torch.bfloat16)
        self.k = torch.randn(self.n, 1, H * D, generator=self.g).to(torch.bfloat16)

    def layer(self) -> float:
        from oracle.attention import forward_with_cache

        t0 = time.perf_counter()
        forward_with_cache(self.store, 0, self.q, self.k, self.k, CFG["hq"])  # layer 0 of 2: pos held
        return time.perf_counter() - t0


class CpuReferenceDecode(_CpuDecodeBase):
    """The reference's own code: ``Attention(Hq, D)`` with its ``PagedKVCache`` (KV heads stored repeated).

    The cache has two layers and the timed calls use layer 0, so ``pos`` is held
    (the reference advances it on the last layer only) and every call sees the
    same contexts.  Runs under ``torch.no_grad`` as the reference engine does.
    """

    kind = "reference"

    def __init__(self, n_sample: int | None = None, threads: int | None = None):
        super().__init__(n_sample, threads)
        mods = _reference_modules()
        if mods is None:
            raise RuntimeError("the reference is not installed in baseline/_ref")
        Attention, RefCache = mods
        Hq, Hkv, D, bs = CFG["hq"], CFG["hkv"], CFG["d"], CFG["bs"]
        G = Hq // Hkv
        cache = RefCache(2, max(self.ctx) + 64, Hq, D, device="cpu", dtype=torch.bfloat16, block_size=bs,
                         enable_prefix_cache=False)
        cache.init_batch(self.n)
        with torch.no_grad():
            for s, c in enumerate(self.ctx):  # through the reference's own append, both layers (not timed)
                kk = torch.randn(c, Hkv, D, generator=self.g).to(torch.bfloat16).repeat_interleave(G, dim=1)
                vv = torch.randn(c, Hkv, D, generator=self.g).to(torch.bfloat16).repeat_interleave(G, dim=1)
                cache.append(s, 0, kk, vv)
                cache.append(s, 1, kk, vv)
        self.cache = cache
        self.attn = Attention(Hq, D)
        self.q = torch.randn(self.n, 1, Hq * D, generator=self.g).to(torch.bfloat16)
        self.k = (torch.randn(self.n, 1, Hkv, D, generator=self.g).to(torch.bfloat16)
                  .repeat_interleave(G, dim=2).reshape(self.n, 1, Hq * D))

    def layer(self) -> float:
        with torch.no_grad():
            t0 = time.perf_counter()
            self.attn(self.q, self.k, self.k, kv_cache=self.cache, layer_id=0)
            return time.perf_counter() - t0


class CpuReferencePrefix(CpuReferenceDecode):
    """The shared-prefix workload on the reference's own code: its PagedKVCache with its prefix cache enabled,
    built the way its engine builds it (try_load_prefix, append the rest, register_prefix; prefix_cache.py:33-81,
    paged_kv_cache.py:87-105), so that sampled requests on the same prefix share its blocks; then decode layers
    through its Attention as in the decode workload."""

    def __init__(self, n_sample: int | None = None, threads: int | None = None):
        _CpuDecodeBase.__init__(self, n_sample, threads)
        mods = _reference_modules()
        if mods is None:
            raise RuntimeError("the reference is not installed in baseline/_ref")
        Attention, RefCache = mods
        Hq, Hkv, D, bs = CFG["hq"], CFG["hkv"], CFG["d"], CFG["bs"]
        G = Hq // Hkv
        prefixes, group, suffix = _prefix_shape(CFG["seqs"])
        population = [CFG["prefix_len"] + len(x) for x in suffix]
        pick = _stratified(population, self.n)
        self.ctx = [population[i] for i in pick]
        cache = RefCache(2, max(self.ctx) + 64, Hq, D, device="cpu", dtype=torch.bfloat16, block_size=bs,
                         enable_prefix_cache=True)
        cache.init_batch(self.n)
        with torch.no_grad():
            for s_, r in enumerate(pick):
                tokens = prefixes[group[r]] + suffix[r]
                matched = cache.try_load_prefix(s_, tokens)
                n_new = len(tokens) - matched
                kk = torch.randn(n_new, Hkv, D, generator=self.g).to(torch.bfloat16).repeat_interleave(G, dim=1)
                vv = torch.randn(n_new, Hkv, D, generator=self.g).to(torch.bfloat16).repeat_interleave(G, dim=1)
                cache.append(s_, 0, kk, vv)
                cache.append(s_, 1, kk, vv)
                cache.register_prefix(s_, tokens)
        # block references beyond the distinct blocks held: the imported (shared) prefix blocks
        self.shared_blocks = int(sum(len(t.physical_blocks()) for t in cache.block_tables) - cache.allocated_blocks)
        self.cache = cache
        self.attn = Attention(Hq, D)
        self.q = torch.randn(self.n, 1, Hq * D, generator=self.g).to(torch.bfloat16)
        self.k = (torch.randn(self.n, 1, Hkv, D, generator=self.g).to(torch.bfloat16)
                  .repeat_interleave(G, dim=2).reshape(self.n, 1, Hq * D))

    def describe(self, calls: int, seconds: float) -> str:
        return super().describe(calls, seconds) + (f"; {self.shared_blocks} block references shared through the "
                                                   "reference prefix cache")


def _time_cpu(make, seconds: float, warmup: int = 1):
    cpu = make()
    for _ in range(warmup):
        cpu.layer()
    times = []
    while sum(times) < seconds or len(times) < 2:
        times.append(cpu.layer())
    t = sum(times) / len(times)
    return {"value": cpu.rate(t), "unit": "tok/s", "cores": torch.get_num_threads(), "host_cpus": os.cpu_count(),
            "kind": cpu.kind, "sample": cpu.describe(len(times), sum(times))}


def cpu_baseline(seconds: float, port_cls, ref_cls, threads: int | None = None):
    """The CPU baseline of a workload: the reference's own code when installed (its value is the line's),
    the oracle port beside it."""
    threads = threads or os.cpu_count() or 1
    port = _time_cpu(lambda: port_cls(threads=threads), seconds)
    ref = None
    if ref_cls is not None and _reference_modules() is not None:
        ref = _time_cpu(lambda: ref_cls(threads=threads), seconds)
        ref["layout"] = f"MHA-expanded: KV heads stored repeated to {CFG['hq']} (the reference has one head count)"
    if ref is None:
        return dict(port, note="reference code not installed in baseline/_ref: the port is the baseline")
    return dict(ref, port=port)


# mixed step on the CPU: one prefill chunk and a sample of the decodes per call, all four chunks in turn
class _CpuMixedBase:
    kind = ""

    def __init__(self, threads: int | None = None):
        if threads:
            torch.set_num_threads(threads)
        prefix, dctx = _mixed_shape()
        self.prefix, self.dctx = prefix, dctx
        self.nd = min(CFG["cpu_sample"], len(dctx))
        self.dsel = _stratified(dctx, self.nd)
        self.ctx = prefix + [dctx[i] for i in self.dsel]  # slots 0..3 chunks, then the sampled decodes
        self.g = torch.Generator().manual_seed(1)
        self.calls = 0

    def rate(self, t_chunk: float, t_dec: float) -> float:
        t_layer = len(self.prefix) * t_chunk + len(self.dctx) / self.nd * t_dec
        tokens = len(self.prefix) * CFG["chunk"] + len(self.dctx)
        return tokens / (CFG["layers"] * t_layer)

    def describe(self, calls: int, seconds: float) -> str:
        return (f"each call one 512-token chunk (the 4 chunks, prefixes {self.prefix}, in turn) and {self.nd} of "
                f"{len(self.dctx)} decodes at evenly spaced context quantiles, one layer x {calls} calls in "
                f"{seconds:.1f} s, scaled to 4 chunks + {len(self.dctx)} decodes x {CFG['layers']} layers")


class CpuOracleMixed(_CpuMixedBase):
    kind = "port"

    def __init__(self, threads: int | None = None):
        from oracle.paged import OracleStore

        super().__init__(threads)
        H, D, bs, C = CFG["hkv"], CFG["d"], CFG["bs"], CFG["chunk"]
        st = OracleStore(2, max(self.ctx) + C + 64, H, D, batch_size=len(self.ctx), dtype=torch.bfloat16,
                         block_size=bs, prefix=False)
        for sl, c in enumerate(self.ctx):
            if c == 0:
                continue
            st.tables[sl].ensure(c)
            kk = torch.randn(c, H, D, generator=self.g).to(torch.bfloat16)
            vv = torch.randn(c, H, D, generator=self.g).to(torch.bfloat16)
            for i, b in enumerate(st.tables[sl].blocks):
                n = min(bs, c - i * bs)
                st.k[0][b, :n] = kk[i * bs: i * bs + n]
                st.v[0][b, :n] = vv[i * bs: i * bs + n]
            st.pos[sl] = c
        self.store = st
        hq = CFG["hq"]
        self.qc = torch.randn(1, C, hq * D, generator=self.g).to(torch.bfloat16)
        self.kc = torch.randn(1, C, H * D, generator=self.g).to(torch.bfloat16)
        self.qd = torch.randn(self.nd, 1, hq * D, generator=self.g).to(torch.bfloat16)
        self.kd = torch.randn(self.nd, 1, H * D, generator=self.g).to(torch.bfloat16)

    def layer(self) -> tuple[float, float]:
        from oracle.attention import forward_with_cache

        c = self.calls % len(self.prefix)
        self.calls += 1
        P = len(self.prefix)
        t0 = time.perf_counter()  # layer 0 of 2: pos held, every call continues the same prefix
        forward_with_cache(self.store, 0, self.qc, self.kc, self.kc, CFG["hq"], slots=[c])
        t1 = time.perf_counter()
        forward_with_cache(self.store, 0, self.qd, self.kd, self.kd, CFG["hq"], slots=list(range(P, P + self.nd)))
        return t1 - t0, time.perf_counter() - t1


class CpuReferenceMixed(_CpuMixedBase):
    kind = "reference"

    def __init__(self, threads: int | None = None):
        super().__init__(threads)
        mods = _reference_modules()
        if mods is None:
            raise RuntimeError("the reference is not installed in baseline/_ref")
        Attention, RefCache = mods
        Hq, Hkv, D, bs, C = CFG["hq"], CFG["hkv"], CFG["d"], CFG["bs"], CFG["chunk"]
        G = Hq // Hkv
        cache = RefCache(2, max(self.ctx) + C + 64, Hq, D, device="cpu", dtype=torch.bfloat16, block_size=bs,
                         enable_prefix_cache=False)
        cache.init_batch(len(self.ctx))

        def rnd(n):
            return torch.randn(n, Hkv, D, generator=self.g).to(torch.bfloat16).repeat_interleave(G, dim=1)

        with torch.no_grad():
            for s, c in enumerate(self.ctx):
                if c:
                    kk, vv = rnd(c), rnd(c)
                    cache.append(s, 0, kk, vv)
                    cache.append(s, 1, kk, vv)
        self.cache = cache
        self.attn = Attention(Hq, D)
        self.qc = torch.randn(1, C, Hq * D, generator=self.g).to(torch.bfloat16)
        self.kc = rnd(C).reshape(1, C, Hq * D)
        self.qd = torch.randn(self.nd, 1, Hq * D, generator=self.g).to(torch.bfloat16)
        self.kd = rnd(self.nd).reshape(self.nd, 1, Hq * D)

    def layer(self) -> tuple[float, float]:
        c = self.calls % len(self.prefix)
        self.calls += 1
        P = len(self.prefix)
        with torch.no_grad():  # layer 0 of 2: pos held, every call continues the same prefix
            t0 = time.perf_counter()
            self.attn(self.qc, self.kc, self.kc, kv_cache=self.cache, layer_id=0, cache_batch_indices=[c])
            t1 = time.perf_counter()
            self.attn(self.qd, self.kd, self.kd, kv_cache=self.cache, layer_id=0,
                      cache_batch_indices=list(range(P, P + self.nd)))
            return t1 - t0, time.perf_counter() - t1


def _time_cpu_mixed(make, seconds: float):
    cpu = make()
    cpu.layer()
    tc, td = [], []
    while sum(tc) + sum(td) < seconds or len(tc) < len(cpu.prefix):
        a, b = cpu.layer()
        tc.append(a)
        td.append(b)
    return {"value": cpu.rate(sum(tc) / len(tc), sum(td) / len(td)), "unit": "tok/s",
            "cores": torch.get_num_threads(), "host_cpus": os.cpu_count(), "kind": cpu.kind,
            "sample": cpu.describe(len(tc), sum(tc) + sum(td))}


def cpu_mixed_baseline(seconds: float, threads: int | None = None):
    threads = threads or os.cpu_count() or 1
    port = _time_cpu_mixed(lambda: CpuOracleMixed(threads=threads), seconds)
    if _reference_modules() is None:
        return dict(port, note="reference code not installed in baseline/_ref: the port is the baseline")
    ref = _time_cpu_mixed(lambda: CpuReferenceMixed(threads=threads), seconds)
    ref["layout"] = f"MHA-expanded: KV heads stored repeated to {CFG['hq']} (the reference has one head count)"
    return dict(ref, port=port)


# ---------------------------------------------------------------------------- GPU helpers
def _dist_setup():
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
    return world, rank, local, dev, dist


def _max_over_ranks(x: float, dev, dist) -> float:
    if dist is None:
        return x
    t = torch.tensor([x], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _check_rows(cache, layer, q, out, checks, group):
    """In-run parity: float32 attention of a few of the step's queries, computed with torch on the GPU
    from the pool (the reference math: softmax(q k^T / sqrt(D)) v over keys [0, pos]), against the
    kernel's output rows.  ``checks``: (slot, q_row, kv_len).  Returns the worst |error| and whether every
    row is within the bf16 tolerance (rtol = atol = 2e-2)."""
    D, bs = cache.head_dim, cache.block_size
    worst, ok = 0.0, True
    for slot, row, kv_len in checks:
        nb = (kv_len + bs - 1) // bs
        idx = torch.tensor(cache.block_tables[slot].physical_blocks()[:nb], device=q.device)
        K = cache.k[layer].index_select(0, idx).reshape(nb * bs, -1, D)[:kv_len].float()
        V = cache.v[layer].index_select(0, idx).reshape(nb * bs, -1, D)[:kv_len].float()
        K = K.repeat_interleave(group, dim=1).transpose(0, 1)
        V = V.repeat_interleave(group, dim=1).transpose(0, 1)
        qs = q[row].view(-1, 1, D).float()
        ref = (torch.softmax((qs @ K.transpose(1, 2)) / math.sqrt(D), dim=-1) @ V).reshape(-1)
        got = out[row].float()
        err = (got - ref).abs()
        worst = max(worst, float(err.max()))
        ok = ok and bool((err <= 2e-2 + 2e-2 * ref.abs()).all())
    return worst, ok


# ---------------------------------------------------------------------------- decode workloads
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


def measure_decode(steps, warmup, e2e_steps, world, rank, local, dev, dist):
    """One decode workload (CFG): timed steps, the attention kernel's roofline, the end-to-end rate and an
    in-run parity check.  Returns the JSON line's fields (the same on every rank; rank 0 prints)."""
    from nifre_b200.sharding import HeadShard

    if CFG["hkv"] % world:
        raise SystemExit(f"--gpus {world} must divide {CFG['hkv']} KV heads")
    shard = HeadShard(world, rank, CFG["hq"], CFG["hkv"], CFG["d"])
    hkv, hq = shard.kv_heads, shard.q_heads
    B = CFG["seqs"] * world if CFG["scaling"] == "weak" else CFG["seqs"]
    ctx = _ctx_lens(B, CFG["seed"])
    steps_total = warmup + steps + e2e_steps + 3
    dt = torch.bfloat16
    if CFG.get("kind") == "prefix":
        cache = _build_prefix_cache(B, ctx, steps_total, hkv, dev, dt)
    else:
        cache = _build_decode_cache(B, ctx, steps_total, hkv, dev, dt, rank)
    try:
        return _run_decode_timed(steps, warmup, e2e_steps, cache, B, ctx, world, rank, local, dev, dist, shard,
                                 hkv, hq)
    finally:
        if cache.exchange is not None:
            torch.cuda.synchronize()
            if dist is not None:
                dist.barrier()
            cache.exchange.close()
            cache.exchange = None
        del cache
        torch.cuda.synchronize()
        torch.cuda.empty_cache()


def _run_decode_timed(steps, warmup, e2e_steps, cache, B, ctx, world, rank, local, dev, dist, shard, hkv, hq):
    from nifre_b200 import Attention

    L, L_model, D, bs = CFG["resident"], CFG["layers"], CFG["d"], CFG["bs"]
    dt = torch.bfloat16
    gd = torch.Generator(device=dev).manual_seed(CFG["seed"] + 1000 + rank)
    q_all = torch.randn(L, B, hq * D, device=dev, dtype=dt, generator=gd)
    k_all = torch.randn(L, B, hkv * D, device=dev, dtype=dt, generator=gd)
    v_all = torch.randn(L, B, hkv * D, device=dev, dtype=dt, generator=gd)
    out_loc = torch.empty(L, B, hq * D, device=dev, dtype=dt)
    slots, ones, rows = list(range(B)), [1] * B, list(range(B))
    stream = torch.cuda.current_stream(dev)
    att_events = []
    # N > 1: the attention kernels store every output row into all ranks' gathered buffers (peer stores
    # over NVLink) and end once all ranks' rows are in place -- the exchange is inside the timed launch
    ex = None
    if world > 1:
        from nifre_b200.sharding import PeerExchange
        ex = PeerExchange(shard, B, dt, dev, slots=2 * L)
        cache.exchange = ex

    def out_of(layer):
        return ex.out(ex.slot_for(layer, cache.steps_closed, L), B) if ex is not None else out_loc[layer]

    def step(rec_layer=-1, fixed=False):
        p = cache.plan(slots, ones, rows, q_heads=hq, fixed_layout=fixed)
        layers(p, rec_layer)
        return p

    def layers(p, rec_layer=-1):
        for layer in range(L):
            o = out_of(layer)
            cache.append_step(layer, k_all[layer], v_all[layer], p)
            record = layer == rec_layer
            if record:
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record(stream)
            cache.attention_step(layer, q_all[layer], p, o, exchange=ex)
            if record:
                e1.record(stream)
                att_events.append((e0, e1, p))

    # The timed steps: each plans on the host (one pack launch) and replays a CUDA graph of its layers' append
    # and attention launches, captured once per plan layout and exchange-buffer parity (the exchange's epoch
    # lives on the device, so replays exchange afresh).  A new layout runs eagerly once, then is captured.
    graphs, seen = {}, set()

    def graph_step():
        p = cache.plan(slots, ones, rows, q_heads=hq, fixed_layout=True)
        key = (p.layout_key, cache.steps_closed % 2)
        g = graphs.get(key)
        if g is not None:
            g.replay()
            cache._close(p)  # the host bookkeeping the captured layers did when they ran
            return p
        if key not in seen:
            seen.add(key)
            layers(p)
            return p
        g = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream(dev)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            with torch.cuda.graph(g, stream=side):
                layers(p)
        stream.wait_stream(side)
        graphs[key] = g
        g.replay()  # the capture launched nothing: run this step
        return p

    for _ in range(4):  # the graphs of both parities captured before the warm-up steps
        graph_step()
    for _ in range(warmup):
        graph_step()
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
    for s in range(steps):
        graph_step()
    e_end.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = _max_over_ranks(e_start.elapsed_time(e_end), dev, dist)
    cache.check_status()
    # the attention launches issued from the host one layer at a time, as the step's eager form runs them:
    # events around one layer per step, a different layer each step (events between every pair of kernels
    # would add a drain per event to the step)
    for s in range(min(L, 8)):
        step(rec_layer=s % L, fixed=True)
    torch.cuda.synchronize()
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
    att_avg_ms = _max_over_ranks(sum(att_ms) / len(att_ms), dev, dist)
    achieved = (sum(att_bytes) / len(att_bytes)) / (att_avg_ms * 1e-3) / 1e9
    peak, peak_kind = _peaks()

    # in-run parity: one more step, then a few of its queries against float32 attention over the pool
    lay = L - 1
    o_last = out_of(lay)
    p = step()
    torch.cuda.synchronize()
    pick = _stratified(p.kv_lens, 6)
    worst, ok = _check_rows(cache, lay, q_all[lay], o_last, [(i, i, int(p.kv_lens[i])) for i in pick], hq // hkv)
    worst = _max_over_ranks(worst, dev, dist)
    ok = _max_over_ranks(0.0 if ok else 1.0, dev, dist) == 0.0

    # the attention launches without the host: the last step's per-layer calls (cascade + decode when the plan
    # has cascade tasks; with the exchange over N GPUs) captured in a CUDA graph and replayed back to back, so
    # that host enqueue gaps are not counted and the launches overlap as programmatic serialization lets them
    kv = int(p.kv_lens.sum())
    nblk = int(((p.kv_lens + bs - 1) // bs).sum())
    g_bytes = (kv - shared) * hkv * D * 2 * 2 + 2 * B * hq * D * 2 + 4 * nblk + 16 * B
    side = torch.cuda.Stream(dev)
    side.wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(side):
        with torch.cuda.graph(graph, stream=side):
            for layer in range(L):
                cache.attention_step(layer, q_all[layer], p, out_of(layer), exchange=ex)
    torch.cuda.synchronize()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    n_rep = 20
    ga, gb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ga.record(stream)
    for _ in range(n_rep):
        graph.replay()
    gb.record(stream)
    torch.cuda.synchronize()
    cache.check_status()
    g_us = _max_over_ranks(ga.elapsed_time(gb), dev, dist) * 1e3 / (n_rep * L)
    g_achieved = g_bytes / (g_us * 1e-6) / 1e9
    del graph

    # e2e through the public drop-in API with host buffers: every step uploads its q/k/v from pinned host
    # memory (one copy per tensor, all layers) and downloads its attention outputs (one copy); uploads and
    # downloads run on their own copy streams into double-buffered device tensors, so a step's copies overlap
    # the neighbouring steps' kernels, as a serving loop that prefetches its next batch does
    e2e = None
    if e2e_steps > 1:
        attn = Attention(hq, D)
        W = world * hq * D
        hq_host = torch.empty(L, B, 1, hq * D, dtype=dt).pin_memory()
        hk_host = torch.empty(L, B, 1, hkv * D, dtype=dt).pin_memory()
        hv_host = torch.empty_like(hk_host).pin_memory()
        ho_host = torch.empty(L, B, 1, W, dtype=dt).pin_memory()
        hq_host.copy_(q_all.view(L, B, 1, -1).cpu())
        hk_host.copy_(k_all.view(L, B, 1, -1).cpu())
        hv_host.copy_(v_all.view(L, B, 1, -1).cpu())
        dev_in = [(torch.empty(L, B, 1, hq * D, device=dev, dtype=dt), torch.empty(L, B, 1, hkv * D, device=dev,
                   dtype=dt), torch.empty(L, B, 1, hkv * D, device=dev, dtype=dt)) for _ in range(2)]
        dev_out = [torch.empty(L, B, 1, W, device=dev, dtype=dt) for _ in range(2)]
        up, down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        ev = lambda: torch.cuda.Event()  # noqa: E731
        consumed = [None, None]  # compute finished reading buffer i (its inputs may be overwritten)
        produced = [None, None]  # compute finished writing buffer i's outputs
        drained = [None, None]   # buffer i's outputs are on the host
        uploaded = [None, None]

        def upload(i):
            with torch.cuda.stream(up):
                if consumed[i] is not None:
                    up.wait_event(consumed[i])
                for d_, h_ in zip(dev_in[i], (hq_host, hk_host, hv_host)):
                    d_.copy_(h_, non_blocking=True)
                uploaded[i] = ev()
                uploaded[i].record(up)

        def compute(i):
            stream.wait_event(uploaded[i])
            if drained[i] is not None:
                stream.wait_event(drained[i])
            qd, kd, vd = dev_in[i]
            outs = []
            for layer in range(L):
                # with N > 1 the cache's exchange makes this the gathered output of every rank's heads
                outs.append(attn(qd[layer], kd[layer], vd[layer], kv_cache=cache, layer_id=layer,
                                 cache_batch_indices=slots))
            torch.stack(outs, out=dev_out[i])
            consumed[i] = ev()
            consumed[i].record(stream)
            produced[i] = consumed[i]

        def download(i):
            with torch.cuda.stream(down):
                down.wait_event(produced[i])
                ho_host.copy_(dev_out[i], non_blocking=True)
                drained[i] = ev()
                drained[i].record(down)

        def run(n):
            upload(0)
            for j in range(n):
                if j + 1 < n:
                    upload((j + 1) % 2)
                compute(j % 2)
                download(j % 2)
            stream.wait_event(drained[(n - 1) % 2])

        run(2)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        up.wait_event(a)
        n_e2e = e2e_steps - 1
        run(n_e2e)
        b.record(stream)
        torch.cuda.synchronize()
        ems = _max_over_ranks(a.elapsed_time(b), dev, dist)
        cache.check_status()
        e2e = {"value": B * n_e2e / (ems * 1e-3) * L / L_model, "unit": "tok/s",
               "h2d_bytes_per_step": L * B * (hq + 2 * hkv) * D * 2,
               "d2h_bytes_per_step": L * B * W * 2,
               "ms_per_step": ems / n_e2e * L_model / L,
               "path": "nifre_b200.Attention.forward per layer; every step's q/k/v copied up from pinned host memory "
                       "(one copy per tensor) and its outputs copied down (one copy) on copy streams, double-buffered "
                       "so that copies overlap the neighbouring steps' kernels; all copies inside the timed region"}

    return {
        "metric": CFG["metric"], "value": B * steps / (ms * 1e-3) * L / L_model, "unit": "tok/s",
        "n_gpus": world, "steps": steps, "warmup": warmup,
        "ms_per_step": ms / steps * L_model / L,
        "higher_is_better": True, "scaling": CFG["scaling"], "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) Q/K/V, random block permutation)",
        "config": {"workload": CFG["name"], "layers": L_model, "layers_timed": L, "q_heads": CFG["hq"],
                   "kv_heads": CFG["hkv"], "head_dim": D, "block_size": bs,
                   "seqs_per_gpu_x_heads": f"{B} seqs x {hkv} kv heads",
                   "global_batch": B,
                   "ctx": (f"U[{CFG['ctx_lo']},{CFG['ctx_hi']}] + step" if "ctx_lo" in CFG else
                           f"{CFG['prefix_len']}-token prefix (one of {CFG['prefixes']}, shared blocks) + "
                           f"U[{CFG['suffix_lo']},{CFG['suffix_hi']}] suffix + step"),
                   "parallelism": (f"kv-head shard x{world}; outputs gathered by the attention kernels' peer "
                                   "stores over NVLink (no collective library call)" if world > 1 else "single GPU"),
                   "method": (("all layers run every step" if L == L_model else
                               f"{L} resident layer(s) run per step; tok/s and ms_per_step scaled to "
                               f"{L_model} layers at the measured per-layer time") +
                              "; a step = plan + pack on the host, then one replay of a CUDA graph of the layers' "
                              "append and attention launches (captured per plan layout)"),
                   "l2": ("inputs larger than L2 (each layer reads a distinct pool of >=300 MB)"
                          if not shared else
                          "each layer reads a distinct pool; shared prefix blocks (16 MB per layer) are read by "
                          "every sequence that imported them: the roofline counts them once (unique bytes)")},
        "roofline": {"bound": "hbm", "achieved": g_achieved, "peak": peak, "unit": "GB/s",
                     "frac": g_achieved / peak,
                     "traffic": (CFG["traffic_ratio"] * sum(att_bytes) / len(att_bytes)
                                 if CFG.get("traffic_ratio") else None),
                     "traffic_source": CFG.get("traffic_source"),
                     "kernel": "nf_paged_attention",
                     "kernel_path": {0: "per-warp cp.async", 1: "tensor map, one copy per block",
                                     2: "tensor map, one copy per head"}.get(att_path, str(att_path)),
                     "peak_source": peak_kind, "avg_launch_us": g_us,
                     "bytes_per_launch": g_bytes,
                     "timing": ("CUDA events around 20 replays of a CUDA graph of one step's per-layer attention "
                                "calls (cascade + decode launches when the step has cascade tasks; the exchange "
                                "over N GPUs), divided by the layers; max over ranks"),
                     "launches_per_layer": 2 if p.n_casc_tasks else 1,
                     "eager": {"avg_launch_us": att_avg_ms * 1e3, "achieved": achieved, "frac": achieved / peak,
                               "what": "events around one layer's attention call per step, the calls issued from "
                                       "the host one layer at a time"},
                     **({"bytes": "unique (shared prefix blocks once)",
                         "achieved_logical": (sum(logical_bytes) / len(logical_bytes)) / (g_us * 1e-6) / 1e9}
                        if shared else {})},
        "parity": {"rows_checked": len(pick) * world, "max_abs_err": worst, "within_tol": ok,
                   "against": "float32 torch attention over the pool, last layer of one extra step",
                   "tol": "rtol 2e-2, atol 2e-2"},
        "e2e": e2e,
        "gpu_launches": steps * (1 + L * (3 if p.n_casc_tasks else 2)),
        "clocks": clk,
    }


# ---------------------------------------------------------------------------- mixed step (prefill + decode)
def measure_mixed(steps, warmup, e2e_steps, world, rank, local, dev, dist):
    """The mixed step (CFG): per layer the KV append, the tensor-core prefill of the 4 chunks and the split-K
    decode, on one plan.  Returns the JSON line's fields."""
    from nifre_b200 import PagedKVCache
    from nifre_b200.sharding import HeadShard

    shard = HeadShard(world, rank, CFG["hq"], CFG["hkv"], CFG["d"])
    hkv, hq = shard.kv_heads, shard.q_heads
    L, D, bs, C = CFG["resident"], CFG["d"], CFG["bs"], CFG["chunk"]
    L_model = CFG["layers"]
    prefix, dctx = _mixed_shape()
    P, ND = len(prefix), len(dctx)
    B = P + ND
    steps_total = warmup + steps + e2e_steps + 3
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
    slots = list(range(B))
    stream = torch.cuda.current_stream(dev)
    kev = []
    ex = None
    if world > 1:  # outputs gathered by the kernels' peer stores (see measure_decode)
        from nifre_b200.sharding import PeerExchange
        ex = PeerExchange(shard, T, dt, dev, slots=2 * L)
        cache.exchange = ex

    def out_of(layer):
        return ex.out(ex.slot_for(layer, cache.steps_closed, L), T) if ex is not None else out_loc[layer]

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
            o = out_of(layer)
            cache.append_step(layer, kd, vd, p)
            ev = None
            if layer == rec_layer:
                ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
                kev.append((ev, p))
            cache.attention_step(layer, qd, p, o, events=ev, exchange=ex)
            if ex is not None and host is not None:  # o is this rank's columns of the gathered rows
                host[3][layer].copy_(o.as_strided((T, ex.width), (ex.width, 1), o.storage_offset() - hq * D * rank),
                                     non_blocking=True)
        if host is not None and world == 1:  # the step's outputs down in one copy
            host[3].copy_(out_loc, non_blocking=True)
        return p

    for _ in range(warmup):
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
    for s in range(steps):
        step(rec_layer=s % L)
    e1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = _max_over_ranks(e0.elapsed_time(e1), dev, dist)
    cache.check_status()
    pre_avg = _max_over_ranks(sum(a[0].elapsed_time(a[1]) for a, _ in kev) / len(kev), dev, dist)
    dec_avg = _max_over_ranks(sum(a[1].elapsed_time(a[2]) for a, _ in kev) / len(kev), dev, dist)
    flops = _mixed_flops(prefix, hq, D, C)  # this rank's heads
    dec_bytes = []
    for _, p in kev:
        kv = p.kv_lens[P:]
        dec_bytes.append(int(kv.sum()) * hkv * D * 4 + 2 * ND * hq * D * 2 + 4 * int(((kv + bs - 1) // bs).sum()))
    hbm_peak, hbm_kind = _peaks()
    tf_burst, tf_sust, tf_kind = _tensor_peaks()

    # in-run parity: one more step; the last 4 queries of every chunk and 8 decodes against float32 attention
    lay = L - 1
    o_last = out_of(lay)
    p = step()
    torch.cuda.synchronize()
    checks = [(i, starts[i] + t, prefix[i] + t + 1) for i in range(P) for t in (C - 4, C - 3, C - 2, C - 1)]
    checks += [(P + i, starts[P + i], int(p.kv_lens[P + i])) for i in _stratified(dctx, 8)]
    worst, ok = _check_rows(cache, lay, q_all[lay], o_last, checks, hq // hkv)
    worst = _max_over_ranks(worst, dev, dist)
    ok = _max_over_ranks(0.0 if ok else 1.0, dev, dist) == 0.0

    # e2e: the same steps through the cache API with q/k/v copied from pinned host memory and the
    # attention output copied back
    e2e = None
    if e2e_steps > 1:
        host = (q_all.cpu().pin_memory(), k_all.cpu().pin_memory(), v_all.cpu().pin_memory(),
                torch.empty(L, T, hq * D * world, dtype=dt).pin_memory())
        step(host=host)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(e2e_steps - 1):
            step(host=host)
        b.record(stream)
        torch.cuda.synchronize()
        ems = _max_over_ranks(a.elapsed_time(b), dev, dist)
        n = e2e_steps - 1
        e2e = {"value": T * n / (ems * 1e-3) * L / L_model, "unit": "tok/s",
               "h2d_bytes_per_step": L * T * (hq + 2 * hkv) * D * 2, "d2h_bytes_per_step": L * T * hq * world * D * 2,
               "ms_per_step": ems / n * L_model / L,
               "path": "PagedKVCache.plan/append_step/attention_step; the step's q/k/v up from pinned host memory in "
                       "one copy per tensor, outputs down in one"}
        cache.check_status()
    if ex is not None:
        torch.cuda.synchronize()
        dist.barrier()
        ex.close()
        cache.exchange = None
    del cache
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    pre_tf = flops * world / (pre_avg * 1e-3) / 1e12
    dec_gbs = (sum(dec_bytes) / len(dec_bytes)) / (dec_avg * 1e-3) / 1e9
    return {
        "metric": CFG["metric"], "value": T * steps / (ms * 1e-3) * L / L_model, "unit": "tok/s", "n_gpus": world,
        "steps": steps, "warmup": warmup, "ms_per_step": ms / steps * L_model / L,
        "higher_is_better": True, "scaling": CFG["scaling"], "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) Q/K/V, random block permutation)",
        "config": {"workload": CFG["name"], "layers": L_model, "layers_timed": L, "q_heads": CFG["hq"],
                   "kv_heads": CFG["hkv"], "head_dim": D, "block_size": bs, "prefill_chunks": P, "chunk_tokens": C,
                   "prefixes": prefix, "decodes": ND, "decode_ctx": f"U[{CFG['dctx_lo']},{CFG['dctx_hi']}]",
                   "tokens_per_step": T, "global_batch": B,
                   "parallelism": (f"kv-head shard x{world}; outputs gathered by the attention kernels' peer "
                                   "stores over NVLink" if world > 1 else "single GPU"),
                   "method": "prefill slots rewound to their prefixes every step; decodes grow by one",
                   "l2": "inputs larger than L2 (each layer reads a distinct pool of ~250 MB)"},
        "roofline": {"bound": "tensor", "achieved": pre_tf, "peak": tf_burst, "unit": "TFLOP/s",
                     "frac": pre_tf / tf_burst, "frac_of_sustained": pre_tf / tf_sust, "traffic": None,
                     "kernel": "nf_prefill_attention",
                     "peak_source": f"{tf_kind} burst (the timed region lasts milliseconds, not seconds)",
                     "avg_launch_us": pre_avg * 1e3, "flops_per_launch": flops * world,
                     "flops_counted": "4*Hq*D per unmasked (query, key) pair"},
        "roofline_decode": {"bound": "hbm", "achieved": dec_gbs, "peak": hbm_peak, "unit": "GB/s",
                            "frac": dec_gbs / hbm_peak, "kernel": "nf_paged_attention",
                            "peak_source": hbm_kind, "avg_launch_us": dec_avg * 1e3},
        "parity": {"rows_checked": len(checks) * world, "max_abs_err": worst, "within_tol": ok,
                   "against": "float32 torch attention over the pool, last layer of one extra step",
                   "tol": "rtol 2e-2, atol 2e-2"},
        "e2e": e2e,
        "gpu_launches": steps * (1 + 3 * L),
        "clocks": clk,
    }


# ---------------------------------------------------------------------------- fused projection + append
def measure_qkv(steps, warmup, world, rank, local, dev, dist):
    """The decode step's input projection fused with the KV append (nf_qkv_append), per layer, against the
    same work as cuBLAS F.linear + nf_kv_append.  Each rank projects its shard's heads (q heads 32/N, KV heads
    8/N) of the full d_model rows.  Returns the JSON line's fields."""
    import torch.nn.functional as F

    from nifre_b200 import PagedKVCache
    from nifre_b200.sharding import HeadShard

    shard = HeadShard(world, rank, CFG["hq"], CFG["hkv"], CFG["d"])
    hkv, hq = shard.kv_heads, shard.q_heads
    L, D, bs, E = CFG["resident"], CFG["d"], CFG["bs"], CFG["d_model"]
    B = CFG["seqs"] * world if CFG["scaling"] == "weak" else CFG["seqs"]
    ctx = _ctx_lens(B, CFG["seed"])
    total = 2 * (warmup + steps) + 8
    dt = torch.bfloat16
    n_blocks = sum((c + total + bs - 1) // bs for c in ctx)
    cache = PagedKVCache(L, max(ctx) + total + 16, hkv, D, device=dev, dtype=dt, block_size=bs,
                         enable_prefix_cache=False, num_blocks=n_blocks)
    cache.init_batch(B)
    g = torch.Generator().manual_seed(CFG["seed"])
    cache.block_allocator.set_free_order(torch.randperm(cache.num_blocks, generator=g).tolist())
    for s_ in range(B):  # contexts allocated (their contents play no part here)
        cache.block_tables[s_].ensure_capacity(ctx[s_])
        cache._set_pos(s_, ctx[s_])
    gd = torch.Generator(device=dev).manual_seed(CFG["seed"] + rank)
    nq, nkv = hq * D, hkv * D
    x = torch.randn(L, B, E, device=dev, dtype=dt, generator=gd)
    w = torch.randn(L, nq + 2 * nkv, E, device=dev, dtype=dt, generator=gd) / math.sqrt(E)
    q = torch.empty(L, B, nq, device=dev, dtype=dt)
    slots, ones, rows = list(range(B)), [1] * B, list(range(B))
    stream = torch.cuda.current_stream(dev)

    def step(fused, rec=None):
        p = cache.plan(slots, ones, rows)
        for layer in range(L):
            if rec is not None and layer == rec[0]:
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
            if fused:
                cache.project_append_step(layer, x[layer], w[layer], None, p, q[layer])
            else:
                y = F.linear(x[layer], w[layer])
                cache.append_step(layer, y[:, nq:nq + nkv], y[:, nq + nkv:], p)
                q[layer].copy_(y[:, :nq])
            if rec is not None and layer == rec[0]:
                e1.record(stream)
                rec[1].append((e0, e1))

    # kernel time without the host: the 16 layers' launches captured in a CUDA graph (one plan's slots reused,
    # pos untouched) and replayed back to back
    from nifre_b200 import _lib
    lib = _lib.load()
    p0 = cache.plan(slots, ones, rows)

    def layers_raw(fused):
        for layer in range(L):
            if fused:
                _lib.check(lib.nf_qkv_append(
                    x[layer].data_ptr(), E, B, w[layer].data_ptr(), None, E, nq, nkv, q[layer].data_ptr(), nq,
                    cache.k[layer].data_ptr(), cache.v[layer].data_ptr(), cache.num_blocks * bs, _lib.NF_BF16,
                    p0.slot_mapping.data_ptr(), None, 0, None, cache.status.data_ptr(), _lib.stream_handle(dev)),
                    "nf_qkv_append")
            else:
                y = F.linear(x[layer], w[layer])
                _lib.check(lib.nf_kv_append(
                    cache.k[layer].data_ptr(), cache.v[layer].data_ptr(), _lib.NF_BF16, cache.num_blocks * bs,
                    y[:, nq:].data_ptr(), y[:, nq + nkv:].data_ptr(), _lib.NF_BF16, y.stride(0), y.stride(0),
                    p0.slot_mapping.data_ptr(), p0.src_rows.data_ptr(), B, hkv, D, p0.seqs.data_ptr(), B, None,
                    cache.status.data_ptr(), _lib.stream_handle(dev)), "nf_kv_append")
                q[layer].copy_(y[:, :nq])

    kern_us = {}
    for fused in (False, True):
        layers_raw(fused)  # warm (cuBLAS handles, function attributes)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            layers_raw(fused)
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(20):
            graph.replay()
        b.record(stream)
        torch.cuda.synchronize()
        kern_us[fused] = _max_over_ranks(a.elapsed_time(b), dev, dist) * 1e3 / (20 * L)
        del graph
    cache._close(p0)

    res = {}
    for fused in (False, True):
        for _ in range(warmup):
            step(fused)
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        ev = []
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for s_ in range(steps):
            step(fused, (s_ % L, ev))
        b.record(stream)
        torch.cuda.synchronize()
        res[fused] = (_max_over_ranks(a.elapsed_time(b), dev, dist),
                      _max_over_ranks(sum(x_.elapsed_time(y_) for x_, y_ in ev) / len(ev), dev, dist))
    cache.check_status()
    # parity of the fused output of the last step's last layer against float32
    ref = x[L - 1].float() @ w[L - 1].float().T
    err = float((q[L - 1].float() - ref[:, :nq]).abs().max())
    ok = bool(torch.allclose(q[L - 1].float(), ref[:, :nq], rtol=1e-2, atol=1e-2))
    ms_f, lay_f = res[True]
    ms_u, lay_u = res[False]
    bytes_layer = (nq + 2 * nkv) * E * 2 + B * E * 2 + B * (nq + 2 * nkv) * 2 + 8 * B
    peak, peak_kind = _peaks()
    del cache
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return {
        "metric": CFG["metric"], "value": B * steps / (ms_f * 1e-3), "unit": "rows/s", "n_gpus": world,
        "steps": steps, "warmup": warmup, "ms_per_step": ms_f / steps, "higher_is_better": True,
        "scaling": CFG["scaling"], "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1))",
        "config": {"workload": CFG["name"], "layers": L, "rows": B, "d_model": E, "q_heads": CFG["hq"],
                   "kv_heads": CFG["hkv"], "head_dim": D, "weight_shape": [nq + 2 * nkv, E],
                   "l2": "a distinct 12.6 MB weight per layer (201 MB over 16 layers): larger than L2",
                   "method": "value: steps through PagedKVCache.plan + project_append_step per layer (host "
                             "included); roofline: kernel time from CUDA-graph replays of the 16 launches",
                   "baseline_path": "torch F.linear (cuBLAS) + nf_kv_append + the q copy",
                   "baseline_ms_per_step": ms_u / steps, "baseline_api_us_per_layer": lay_u * 1e3,
                   "baseline_kernels_us_per_layer": kern_us[False], "fused_api_us_per_layer": lay_f * 1e3},
        "roofline": {"bound": "hbm", "achieved": bytes_layer / (kern_us[True] * 1e-6) / 1e9, "peak": peak,
                     "unit": "GB/s", "frac": bytes_layer / (kern_us[True] * 1e-6) / 1e9 / peak, "traffic": None,
                     "kernel": "nf_qkv_append", "peak_source": peak_kind, "avg_launch_us": kern_us[True],
                     "bytes_per_launch": bytes_layer, "bytes": "weights + x rows + q/k/v outputs + slots"},
        "parity": {"max_abs_err": err, "within_tol": ok, "against": "float32 x W^T", "tol": "rtol 1e-2, atol 1e-2"},
        "gpu_launches": steps * (1 + L),
    }


# ---------------------------------------------------------------------------- arms
def _sub_result(line: dict) -> dict:
    keep = ("metric", "value", "unit", "ms_per_step", "steps", "warmup", "dtype", "config", "roofline",
            "roofline_decode", "parity", "cpu_baseline", "e2e", "clocks")
    return {k: line[k] for k in keep if k in line}


def run_ours(args):
    world, rank, local, dev, dist = _dist_setup()
    kind = CFG.get("kind")
    # the CPU baselines run on rank 0 at N = 1 only (the other arm times the reference at every N)
    args.no_cpu_baseline = args.no_cpu_baseline or world > 1
    if kind == "engine":
        line = measure_engine(args, world, rank, local, dev, dist)
    elif kind == "qkv":
        line = measure_qkv(args.steps, args.warmup, world, rank, local, dev, dist)
    elif kind == "mixed":
        line = measure_mixed(args.steps, args.warmup, args.e2e_steps, world, rank, local, dev, dist)
        if rank == 0 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_mixed_baseline(12.0)
    else:
        line = measure_decode(args.steps, args.warmup, args.e2e_steps, world, rank, local, dev, dist)
        if rank == 0 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(12.0, CpuOracleDecode,
                                                CpuReferencePrefix if kind == "prefix" else CpuReferenceDecode)
    if CFG["name"] == "llama3.2-1b-decode" and not args.no_sub and not args.layers and not args.seqs:
        subs = {}
        for name, resident, steps in SUB_RESULTS:
            with _workload(name, resident=resident):
                sub_kind = CFG.get("kind")
                if sub_kind == "engine":
                    sub = measure_engine(argparse.Namespace(steps=steps, warmup=2,
                                                            no_cpu_baseline=args.no_cpu_baseline),
                                         world, rank, local, dev, dist)
                elif sub_kind == "qkv":
                    sub = measure_qkv(steps, 3, world, rank, local, dev, dist)
                elif sub_kind == "mixed":
                    sub = measure_mixed(steps, 3, 0, world, rank, local, dev, dist)
                    if rank == 0 and not args.no_cpu_baseline:
                        sub["cpu_baseline"] = cpu_mixed_baseline(8.0)
                else:
                    sub = measure_decode(steps, 3, 0, world, rank, local, dev, dist)
                    if rank == 0 and not args.no_cpu_baseline:
                        sub["cpu_baseline"] = cpu_baseline(
                            8.0, CpuOracleDecode, CpuReferencePrefix if sub_kind == "prefix" else CpuReferenceDecode)
                subs[name] = _sub_result(sub)
                line["gpu_launches"] += sub["gpu_launches"]
        line["sub_results"] = subs
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def _reference_qkv(args, world, threads, use_ref):
    """The projection + append on the host cores: the three nn.Linear projections of the reference's
    GptAttention (models/gpt.py:38-51, torch's CPU GEMM) and its PagedKVCache.append of the new k/v rows
    (paged_kv_cache.py:107-121, the reference's own code when installed), one layer per call."""
    torch.set_num_threads(threads)
    Hq, Hkv, D, E, B = CFG["hq"], CFG["hkv"], CFG["d"], CFG["d_model"], CFG["seqs"]
    g = torch.Generator().manual_seed(1)
    x = torch.randn(B, E, generator=g).to(torch.bfloat16)
    wq = (torch.randn(Hq * D, E, generator=g) / math.sqrt(E)).to(torch.bfloat16)
    wk = (torch.randn(Hkv * D, E, generator=g) / math.sqrt(E)).to(torch.bfloat16)
    wv = (torch.randn(Hkv * D, E, generator=g) / math.sqrt(E)).to(torch.bfloat16)
    ctx = _ctx_lens(B, CFG["seed"])
    if use_ref:
        _, RefCache = _reference_modules()
        cache = RefCache(2, max(ctx) + args.steps + args.warmup + 8, Hkv, D, device="cpu", dtype=torch.bfloat16,
                         block_size=CFG["bs"], enable_prefix_cache=False)
        cache.init_batch(B)
        for s_ in range(B):
            cache.block_tables[s_].ensure_capacity(ctx[s_])
            cache.pos[s_] = ctx[s_]
        kind = "reference"
    else:
        from oracle.paged import OracleStore
        cache = OracleStore(2, max(ctx) + args.steps + args.warmup + 8, Hkv, D, batch_size=B, dtype=torch.bfloat16,
                            block_size=CFG["bs"], prefix=False)
        for s_ in range(B):
            cache.tables[s_].ensure(ctx[s_])
            cache.pos[s_] = ctx[s_]
        kind = "port"
    F = torch.nn.functional

    def layer():
        t0 = time.perf_counter()
        with torch.no_grad():
            qq, kk, vv = F.linear(x, wq), F.linear(x, wk), F.linear(x, wv)
            for s_ in range(B):  # layer 0 of 2: pos held
                cache.append(s_, 0, kk[s_].view(1, Hkv, D), vv[s_].view(1, Hkv, D))
        return time.perf_counter() - t0

    for _ in range(args.warmup):
        layer()
    times = [layer() for _ in range(args.steps)]
    v = B / (CFG["layers"] * sum(times) / len(times))  # rows of 16-layer steps per second
    base = {"value": v, "unit": "rows/s", "cores": torch.get_num_threads(), "host_cpus": os.cpu_count(), "kind": kind,
            "sample": f"the {B} rows of one layer x {len(times)} calls in {sum(times):.1f} s, scaled to "
                      f"{CFG['layers']} layers; each step = one call"}
    return {"impl": "reference", "metric": METRIC, "value": v, "unit": "rows/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": True, "scaling": CFG["scaling"], "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic", "config": {"workload": CFG["name"], "d_model": E, "rows": B},
            "cpu_baseline": base, "e2e": {"value": v, "unit": "rows/s", "h2d_bytes_per_step": 0,
                                          "d2h_bytes_per_step": 0}}


def run_reference(args):
    """The reference's CPU path on the host cores (rank 0 alone; other ranks exit without work)."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    if CFG.get("kind") == "engine":
        seconds = max(5.0, 1.0 * args.steps / 10)
        cpu = cpu_engine_reference_rate(seconds, threads=threads)
        if cpu is None:
            cpu = dict(cpu_engine_rate(seconds, threads=threads), kind="port", host_cpus=os.cpu_count())
        line = {"impl": "reference", "metric": METRIC, "value": cpu["value"], "unit": "tok/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": CFG["scaling"],
                "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
                "config": {"workload": CFG["name"], "model": "GPT-124M (12 layers, 12 heads, d 64, context 2048)"},
                "cpu_baseline": cpu,
                "e2e": {"value": cpu["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return
    use_ref = _reference_modules() is not None
    if CFG.get("kind") == "qkv":
        line = _reference_qkv(args, world, threads, use_ref)
        print(json.dumps(line), flush=True)
        return
    if CFG.get("kind") == "mixed":
        cpu = (CpuReferenceMixed if use_ref else CpuOracleMixed)(threads=threads)
        for _ in range(args.warmup):
            cpu.layer()
        pairs = [cpu.layer() for _ in range(args.steps)]
        v = cpu.rate(sum(a for a, _ in pairs) / len(pairs), sum(b for _, b in pairs) / len(pairs))
        times = [a + b for a, b in pairs]
    else:
        ref_cls = CpuReferencePrefix if CFG.get("kind") == "prefix" else CpuReferenceDecode
        cpu = (ref_cls if use_ref else CpuOracleDecode)(threads=threads)
        for _ in range(args.warmup):
            cpu.layer()
        times = [cpu.layer() for _ in range(args.steps)]
        v = cpu.rate(sum(times) / len(times))
    base = {"value": v, "unit": "tok/s", "cores": torch.get_num_threads(), "host_cpus": os.cpu_count(),
            "kind": cpu.kind, "sample": cpu.describe(len(times), sum(times)) + "; each step = one such call"}
    if use_ref:
        base["layout"] = f"MHA-expanded: KV heads stored repeated to {CFG['hq']} (the reference has one head count)"
        base["code"] = "reference src/inference/attention.py + paged_kv_cache.py, installed unmodified in baseline/_ref"
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": CFG["scaling"],
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": CFG["name"], "layers": CFG["layers"], "q_heads": CFG["hq"],
                       "kv_heads": CFG["hkv"], "head_dim": CFG["d"], "block_size": CFG["bs"]},
            "cpu_baseline": base,
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


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


def cpu_engine_reference_rate(seconds: float, threads: int | None = None):
    """The reference's own Engine with its own GPT-124M (random init, seed 0, fp32, context 2048) on the host
    cores, generating the workload's 8 requests through add_request/step (tokens counted by its token
    callbacks): tok/s over whole generations, prefill included, as the GPU engine's value is; bounded at about
    ``seconds`` of steps."""
    if _reference_modules() is None:
        return None
    from inference.backends.gpt import GptInferenceModel as RefInferenceModel
    from inference.engine import Engine as RefEngine
    from inference.models.gpt import GPT_CONFIG_124M as REF_CFG
    from inference.models.gpt import GptModel as RefGptModel
    if threads:
        torch.set_num_threads(threads)
    torch.manual_seed(CFG["seed"])
    model = RefGptModel(dict(REF_CFG, context_length=2048)).eval()
    eng = RefEngine(RefInferenceModel(model), max_concurrent_requests=CFG["requests"], device=torch.device("cpu"),
                    prefill_chunk_size=128, max_tokens_per_step=2048)
    count = [0]

    def on_token(_tok):
        count[0] += 1

    for prompt in _engine_prompts(CFG["seed"]):
        eng.register_token_callback(eng.add_request(prompt, CFG["new_tokens"]), on_token)
    steps, t0 = 0, time.perf_counter()
    with torch.no_grad():
        while eng.step():
            steps += 1
            if time.perf_counter() - t0 >= seconds:
                break
    spent = time.perf_counter() - t0
    return {"value": count[0] / spent, "unit": "tok/s", "cores": torch.get_num_threads(),
            "host_cpus": os.cpu_count(), "kind": "reference",
            "sample": f"the workload's {CFG['requests']} requests through the reference Engine: {steps} steps, "
                      f"{count[0]} tokens in {spent:.1f} s (prefill included)",
            "code": "reference src/inference/engine.py + models/gpt.py, installed unmodified in baseline/_ref"}


def cpu_engine_baseline(seconds: float, threads: int | None = None):
    threads = threads or os.cpu_count() or 1
    port = dict(cpu_engine_rate(seconds, threads=threads), kind="port", host_cpus=os.cpu_count())
    ref = cpu_engine_reference_rate(seconds, threads=threads)
    if ref is None:
        return dict(port, note="reference code not installed in baseline/_ref: the port is the baseline")
    return dict(ref, port=port)


def measure_engine(args, world, rank, local, dev, dist):
    """Greedy generation through the engine: every timed step is one Engine.step() (host scheduling, one
    upload of the step's ids/positions, the flat forward, one download of the sampled tokens); N GPUs run N
    independent replicas.  Returns the JSON line's fields (rank 0's)."""
    from nifre_b200 import Engine, GptInferenceModel
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
    if True:
        cpu = None
        if rank == 0 and not args.no_cpu_baseline:
            cpu = cpu_engine_baseline(12.0)
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
    del eng, cache
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return line


def main():
    args = _args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
