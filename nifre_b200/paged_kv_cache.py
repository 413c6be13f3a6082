"""Paged KV cache on B200 HBM (drop-in for nifre's PagedKVCache).

Public API and attributes follow jyotilakra92/nifre
``src/inference/paged_kv_cache.py:8-169`` (``init_batch``, ``append``, ``get``,
``length``, ``lengths``, ``reset_slot``, ``free``, ``try_load_prefix``,
``register_prefix``, ``pos``, ``k``, ``v``, ``block_tables``,
``block_allocator``, ``prefix_cache``, ``num_blocks`` ...), so the engine, the
model runner and the observability probe keep working unchanged.  The pools
keep the reference layout ``(num_blocks, block_size, n_heads, head_dim)`` per
layer, with ``n_heads`` the number of KV heads stored (grouped-query models
store fewer KV heads than they have query heads).

What changes is where the work happens:

* block allocation stays on the host (``BlockAllocator``/``BlockTable``, same
  ids as the reference), but a step's allocations are collected into a
  *step plan*: one int32 upload (sequence records + block-table patches) and
  one ``nf_pack_step`` launch compute every token's destination row, source
  row, position and the split-K work list on the GPU;
* ``append`` is one ``nf_kv_append`` launch for all sequences of the step;
* attention reads K/V in place from the pools (``nf_paged_attention``); the
  ``get`` gather is kept for API compatibility only.

``pos`` stays a device int64 tensor like the reference; a host copy drives
planning so no step ever reads it back.  As in the reference, ``pos``
advances only when the last layer of a step has appended
(``paged_kv_cache.py:120-121``).
"""

from __future__ import annotations

import ctypes
import math

import numpy as np
import torch

from nifre_b200 import _lib
from nifre_b200.block_allocator import BlockAllocator
from nifre_b200.block_table import BlockTable
from nifre_b200.prefix_cache import PrefixCache


class _DeviceBuffer:
    """Grow-only device buffer reused across steps (stream-ordered reuse)."""

    def __init__(self, dtype: torch.dtype, device, zero: bool = False):
        self.dtype, self.device, self.zero = dtype, device, zero
        self.t: torch.Tensor | None = None

    def get(self, n: int) -> torch.Tensor:
        if self.t is None or self.t.numel() < n:
            cap = max(n, int((self.t.numel() if self.t is not None else 0) * 1.5), 64)
            alloc = torch.zeros if self.zero else torch.empty
            self.t = alloc(cap, dtype=self.dtype, device=self.device)
        return self.t


def seq_unit_sizes(seq_keys: np.ndarray, split: int, sms: int, fine_div: int = 4) -> np.ndarray:
    """Split-K unit size of each sequence of a step.

    The bulk of the step uses ``split`` keys per unit.  The shortest
    sequences that together hold at least one wave of units (``sms * split``
    keys) use ``split / fine_div`` (a multiple of 16); nf_pack_step lists their
    units after all others, so a dynamic queue ends on short units and the
    workers finish close together, while being short keeps their split-K
    merges cheap.  Steps with under two waves of keys use ``split``
    throughout.
    """
    seq_keys = np.asarray(seq_keys, dtype=np.int64)
    sizes = np.full(len(seq_keys), split, dtype=np.int32)
    fine = max(16, (split // fine_div) // 16 * 16)
    wave = sms * split
    if fine >= split or int(seq_keys.sum()) < 2 * wave:
        return sizes
    order = np.argsort(seq_keys, kind="stable")  # shortest first
    n_fine = int(np.searchsorted(np.cumsum(seq_keys[order]), wave)) + 1
    sizes[order[:n_fine]] = fine
    return sizes


def _prefill_order(tiles, kv_heads: int) -> np.ndarray:
    """The order in which the prefill kernel's CTAs take its (tile, KV head) items.

    An item costs its 128-key tiles plus one (query load and epilogue).  CTAs
    take items from one shared queue as they free up, so listing the items by
    decreasing cost gives the longest-processing-time-first schedule, adapted
    at run time to the real per-item times.  Returns int32 item numbers
    (tile * kv_heads + head).
    """
    costs = np.asarray([(pos0 + ntok + 127) // 128 + 1 for (_, _, ntok, pos0) in tiles], dtype=np.int64)
    items = np.arange(len(tiles) * kv_heads, dtype=np.int64)
    return items[np.argsort(-costs[items // kv_heads], kind="stable")].astype(np.int32)


class StepPlan:
    """Device metadata of one forward pass over a ragged batch.

    Valid for every layer of that forward; ``PagedKVCache`` closes it when the
    last layer has appended.
    """

    def __init__(self, slots, q_lens, q_starts, ctx_before, split, max_units, seq_split=None):
        self.slots = slots
        self.q_lens = q_lens
        self.q_starts = q_starts
        self.ctx_before = ctx_before
        self.n_seqs = len(slots)
        self.n_tokens = int(q_lens.sum())
        self.rows_needed = int((q_starts + q_lens).max())
        self.split = split
        self.seq_split = seq_split  # unit size of each sequence (numpy)
        self.max_units = max_units
        self.key = None
        self.closed = False
        # device views, filled by PagedKVCache.plan
        self.seqs = self.slot_mapping = self.src_rows = self.items = self.units = self.counts = None
        self.positions = None
        # split-K units of the step, and the tensor-core prefill tiles (tiles, n_tiles, q_heads)
        self.decode_units = max_units
        self.shared_keys = None  # per sequence: leading keys served by the cascade kernel (numpy)
        self.ws_sizes = None  # (query heads, partial floats, counter ints) of the split-K workspace
        self.upload_bytes = 0  # bytes of the step's host-to-device metadata copy
        self.n_casc_tasks = self.n_casc_toks = 0
        self.casc_tasks = self.casc_toks = None  # device: (slot, first, count, part, k0, k1, 0, 0), (item, q row)
        self.tiles = None
        self.n_tiles = 0
        self.q_heads = None
        self.sched = None
        # per-plan constant arguments of the layers' C ABI calls, built on first use
        self.append_args = self.decode_args = None

    @property
    def kv_lens(self) -> np.ndarray:
        return self.ctx_before + self.q_lens


class PagedKVCache:
    def __init__(self, num_layers: int, max_seq_len: int, n_heads: int, head_dim: int,
                 device="cuda", dtype: torch.dtype = torch.float16, block_size: int = 16,
                 enable_prefix_cache: bool = True, prefix_cache_max_entries: int = 1024,
                 num_blocks: int | None = None) -> None:
        if block_size <= 0:
            raise ValueError(f"block_size must be positive, got {block_size}")
        self.num_layers = num_layers
        self.max_seq_len = max_seq_len
        self.n_heads = n_heads
        self.head_dim = head_dim
        self.device = torch.device(device)
        self.dtype = dtype
        self.block_size = block_size
        self.enable_prefix_cache = enable_prefix_cache
        # decode sequences that share leading blocks get those keys attended once per group (cascade)
        self.enable_cascade = True
        self._cascade_memo = None  # (batch key, grouping) of the last step planned
        self._cascade_limit_memo = {}  # query heads per KV head -> cascade_limits()
        self.prefix_cache_max_entries = prefix_cache_max_entries
        self._num_blocks_override = num_blocks
        self.batch_size = 0
        self.num_blocks = 0
        self.pos = None
        self.k = None
        self.v = None
        self.block_allocator: BlockAllocator | None = None
        self.block_tables: list[BlockTable] = []
        self.prefix_cache: PrefixCache | None = None
        self._plan: StepPlan | None = None
        self.steps_closed = 0  # forward passes whose last layer has appended
        # KV heads sharded over several GPUs: a sharding.PeerExchange whose gathered buffers receive every
        # rank's attention output (Attention.forward then returns the gathered rows); None on one GPU
        self.exchange = None

    # ------------------------------------------------------------------ setup
    def init_batch(self, batch_size: int) -> None:
        _lib.load()
        if self.device.type != "cuda":
            raise _lib.NifreError("PagedKVCache needs a CUDA device: nifre_b200 has no CPU path")
        self.batch_size = batch_size
        self.pos = torch.zeros(batch_size, dtype=torch.long, device=self.device)
        self.pos_host = np.zeros(batch_size, dtype=np.int64)
        self.max_blocks_per_seq = (self.max_seq_len + self.block_size - 1) // self.block_size
        self.num_blocks = (self._num_blocks_override if self._num_blocks_override is not None
                           else self.max_blocks_per_seq * batch_size)
        self.block_allocator = BlockAllocator(self.num_blocks)
        self.block_tables = [BlockTable(self.block_allocator, self.block_size) for _ in range(batch_size)]
        self.prefix_cache = (PrefixCache(self.block_allocator, self.block_size,
                                         max_entries=self.prefix_cache_max_entries)
                             if self.enable_prefix_cache else None)
        shape = (self.num_layers, self.num_blocks, self.block_size, self.n_heads, self.head_dim)
        self._k_all = torch.empty(shape, device=self.device, dtype=self.dtype)
        self._v_all = torch.empty(shape, device=self.device, dtype=self.dtype)
        self.k = list(self._k_all.unbind(0))
        self.v = list(self._v_all.unbind(0))
        # per-call constants of the C ABI calls (pointers, codes), so that a layer's launches cost little host time
        self._k_ptr = [t.data_ptr() for t in self.k]
        self._v_ptr = [t.data_ptr() for t in self.v]
        self._dt_code = _lib.dtype_code(self.dtype)
        self._pool_rows = self.num_blocks * self.block_size
        self._row_width = self.n_heads * self.head_dim
        self.bt_dev = torch.zeros((batch_size, self.max_blocks_per_seq), dtype=torch.int32, device=self.device)
        # per slot: the table epoch and the number of entries mirrored on the device
        self._sync_epoch = np.full(batch_size, -1, dtype=np.int64)
        self._sync_len = np.zeros(batch_size, dtype=np.int64)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._status_ptr = self.status.data_ptr()
        self._bt_ptr = self.bt_dev.data_ptr()
        self._pos_ptr = self.pos.data_ptr()
        self._dev_index = self.device.index if self.device.index is not None else torch.cuda.current_device()
        self._pf_queue = torch.zeros(2, dtype=torch.int32, device=self.device)  # prefill work queue (kernel-reset)
        self._meta = _DeviceBuffer(torch.int32, self.device)
        self._pos_buf = _DeviceBuffer(torch.int64, self.device)
        self._ws_partials = _DeviceBuffer(torch.float32, self.device)
        self._ws_counters = _DeviceBuffer(torch.int32, self.device, zero=True)
        self._plan = None

    def free(self) -> None:
        self.batch_size = 0
        self.num_blocks = 0
        self.pos = None
        self.k = None
        self.v = None
        self.block_allocator = None
        self.block_tables = []
        self.prefix_cache = None
        self._plan = None
        self._k_all = self._v_all = None

    # ------------------------------------------------------------------ reference API
    def try_load_prefix(self, batch_idx: int, token_ids: list[int]) -> int:
        if self.prefix_cache is None:
            return 0
        num_tokens, blocks = self.prefix_cache.lookup(token_ids)
        if num_tokens == 0:
            return 0
        self.block_tables[batch_idx].import_blocks(blocks)
        self._set_pos(batch_idx, num_tokens)
        return num_tokens

    def register_prefix(self, batch_idx: int, token_ids: list[int]) -> None:
        if self.prefix_cache is None:
            return
        self.prefix_cache.insert(token_ids, self.block_tables[batch_idx].physical_blocks())

    def append(self, batch_idx: int, layer_id: int, key: torch.Tensor, value: torch.Tensor) -> None:
        """Append ``key``/``value`` (n, H, D) of one sequence (reference per-row API)."""
        n = key.shape[0]
        plan = self.plan([batch_idx], [n], [0])
        self.append_step(layer_id, key.reshape(n, -1), value.reshape(n, -1), plan)

    def get(self, batch_idx: int, layer_id: int) -> tuple[torch.Tensor, torch.Tensor]:
        pos = int(self.pos_host[batch_idx])
        if pos == 0:
            empty = torch.empty(0, self.n_heads, self.head_dim, device=self.device, dtype=self.dtype)
            return empty, empty.clone()
        nb = (pos + self.block_size - 1) // self.block_size
        idx = torch.tensor(self.block_tables[batch_idx].physical_blocks()[:nb], device=self.device)
        k = self.k[layer_id].index_select(0, idx).reshape(-1, self.n_heads, self.head_dim)[:pos]
        v = self.v[layer_id].index_select(0, idx).reshape(-1, self.n_heads, self.head_dim)[:pos]
        return k, v

    def length(self, batch_idx: int) -> int:
        return int(self.pos_host[batch_idx])

    def lengths(self) -> torch.Tensor:
        return self.pos.clone()

    def reset_slot(self, batch_idx: int) -> None:
        self.block_tables[batch_idx].clear()
        self._set_pos(batch_idx, 0)

    @property
    def allocated_blocks(self) -> int:
        return 0 if self.block_allocator is None else self.block_allocator.allocated_count

    def _stream(self) -> int:
        raw = _lib._raw_stream
        return raw(self._dev_index) if raw is not None else _lib.stream_handle(self.device)

    def _set_pos(self, slot: int, value: int) -> None:
        self.pos_host[slot] = value
        self.pos[slot] = value

    # ------------------------------------------------------------------ step planning
    @property
    def sm_count(self) -> int:
        if getattr(self, "_sm_count", None) is None:
            self._sm_count = torch.cuda.get_device_properties(self.device).multi_processor_count
        return self._sm_count

    @property
    def decode_workers(self) -> int:
        """Decode CTAs the attention kernel keeps resident: one group of KV heads each.

        A CTA covers up to 8 KV heads (4 for head_dim 128); with fewer heads in
        the pool (one GPU's shard of the heads) the kernel runs proportionally
        more, smaller CTAs per SM, and the split-K units are sized for them.
        """
        max_hg = 8 if self.head_dim == 64 else 4
        hg = max(h for h in range(1, min(self.n_heads, max_hg) + 1) if self.n_heads % h == 0)
        return self.sm_count * (max_hg // hg)

    def split_for(self, total_keys: int, units_per_sm: int = 4) -> int:
        """Keys per split-K unit.

        Tensor-map kernel (16-bit pools, head_dim 64/128, blocks of a multiple
        of 16): ~units_per_sm units per SM (per decode CTA when the pool holds
        few KV heads), a multiple of 128.  Per-warp kernel (float32 and other
        shapes), where one warp takes one (unit, KV head) and walks its keys
        serially: about two such items per resident warp (64 per SM), a
        multiple of 32, so that small batches spread over the GPU.
        """
        if self.dtype in (torch.bfloat16, torch.float16) and self.head_dim in (64, 128) \
                and self.block_size % 16 == 0:
            s = total_keys / max(1, units_per_sm * self.decode_workers)
            return max(128, int(math.ceil(s / 128.0)) * 128)
        s = total_keys * self.n_heads / max(1, 64 * self.sm_count)
        return max(32, int(math.ceil(s / 32.0)) * 32)

    # sequences with at least this many new tokens go to the tensor-core prefill kernel
    PREFILL_MIN_TOKENS = 16

    def prefill_supported(self, q_heads: int | None) -> bool:
        """True when nf_prefill_attention serves this cache with q_heads query heads."""
        if q_heads is None or q_heads % self.n_heads:
            return False
        return (self.dtype in (torch.bfloat16, torch.float16) and self.head_dim in (64, 128)
                and q_heads // self.n_heads in (1, 2, 4, 8) and self.block_size % 16 == 0)

    # cascade over shared keys: at least this many shared keys and two sequences
    CASCADE_MIN_KEYS = 64
    # the mma.sync cascade kernel (group sizes the tensor-core path does not take): 128 query rows and at most
    # 256 keys per task, two CTAs per SM aimed for
    CASCADE_ROWS = 128
    CASCADE_MAX_KEYS = 256
    CASCADE_WAVES = 2
    # the tensor-core path: one (task, KV head) item per SM aimed for, each at least this many keys long
    CASCADE_TC_MIN_KEYS = 256
    # own keys (in units of the step's split) up to which a cascade sequence's own keys are one decode unit
    CASCADE_OWN_UNIT_MAX = 4

    def cascade_supported(self, q_heads: int | None) -> bool:
        """True when nf_cascade_attention serves this cache with q_heads query heads."""
        if not self.enable_cascade or q_heads is None or q_heads % self.n_heads:
            return False
        return (self.dtype in (torch.bfloat16, torch.float16) and self.head_dim in (64, 128)
                and q_heads // self.n_heads <= self.CASCADE_ROWS and self.block_size % 16 == 0)

    def cascade_limits(self, group: int) -> tuple[int, int, bool]:
        """(query rows, keys) of the largest nf_cascade_attention task for ``group`` query heads per KV head,
        and whether the tasks run on the tensor cores."""
        memo = self._cascade_limit_memo
        if group not in memo:
            rows, keys = ctypes.c_int32(0), ctypes.c_int32(0)
            _lib.check(_lib.load().nf_cascade_limits(_lib.dtype_code(self.dtype), group * self.n_heads, self.n_heads,
                                                     self.head_dim, self.block_size, ctypes.byref(rows),
                                                     ctypes.byref(keys)), "nf_cascade_limits")
            memo[group] = (rows.value, keys.value, keys.value > self.CASCADE_MAX_KEYS)
        return memo[group]

    def _cascade_groups(self, slots, q_lens, q_starts, ctx, dec, group: int, epochs=None):
        """Decode sequences that start with the same physical blocks, and the cascade work over those keys.

        Sequences with one new token whose tables begin with the same block
        are grouped; a group's shared keys are the blocks all its members
        hold at the same positions (imported prefix blocks: full, written
        before the step).  Members are cut into CTA groups of at most
        ``CASCADE_ROWS / group`` sequences (at least two each) and each
        group's shared keys into near-equal ranges of whole 16-key tiles, at
        most ``CASCADE_MAX_KEYS`` keys, with ranges handed out in proportion
        to the groups' shared keys so that (range, KV head) CTAs number about
        ``CASCADE_WAVES`` per SM.  Returns per-sequence shared keys and
        cascade part counts, the (slot, first, count, part, key_begin,
        key_end, 0, 0) tasks and the (item, q row) query records for
        ``nf_cascade_attention``.
        """
        S, bs = len(slots), self.block_size
        # Decode steps repeat the same batch: while its sequences, their new
        # token counts and their tables' epochs (which change only when
        # leading entries are replaced) are those of the previous step, the
        # shared runs are unchanged and the previous grouping stands.
        if epochs is None:
            epochs = np.fromiter((self.block_tables[s].epoch for s in slots.tolist()), np.int64, len(slots))
        key = (slots.tobytes(), q_lens.tobytes(), q_starts.tobytes(), dec.tobytes(), group, epochs.tobytes())
        if (self._cascade_memo is not None and self._cascade_memo[0] == key
                and (self._cascade_memo[1][0] <= ctx).all()):  # no position moved back under a shared run
            return self._cascade_memo[1]
        shared = np.zeros(S, dtype=np.int32)
        nparts = np.zeros(S, dtype=np.int32)
        buckets: dict[int, list[int]] = {}
        for i in np.flatnonzero(dec & (q_lens == 1)).tolist():
            if int(ctx[i]) // bs * bs < self.CASCADE_MIN_KEYS:
                continue
            blocks = self.block_tables[int(slots[i])]._physical_blocks
            buckets.setdefault(blocks[0], []).append(i)
        max_rows, max_keys, tensor_cores = self.cascade_limits(group)
        per_cta = max_rows // group
        cuts = []  # (members, shared keys)
        for members in buckets.values():
            if len(members) < 2:
                continue
            n = min(int(ctx[i]) // bs for i in members)
            ref = self.block_tables[int(slots[members[0]])]._physical_blocks
            for i in members[1:]:
                other = self.block_tables[int(slots[i])]._physical_blocks
                if other[:n] != ref[:n]:
                    n = int(np.argmin(np.asarray(ref[:n]) == np.asarray(other[:n])))
            if n * bs < self.CASCADE_MIN_KEYS:
                continue
            for c0 in range(0, len(members), per_cta):
                part = members[c0: c0 + per_cta]
                if len(part) >= 2:
                    cuts.append((part, n * bs))
        tasks, toks = [], []
        if cuts:
            total = sum(p for _, p in cuts)
            waves = 1 if tensor_cores else self.CASCADE_WAVES
            want = max(len(cuts), round(waves * self.sm_count / self.n_heads))
            tok_off = np.cumsum(q_lens) - q_lens
            for members, p in cuts:
                tiles = p // 16
                nc = max(1, round(want * p / total), -(-p // max_keys))
                if tensor_cores:  # a tensor-core item has a fixed cost: keep parts at least this long
                    nc = max(1, min(nc, p // self.CASCADE_TC_MIN_KEYS))
                nc = min(nc, tiles)
                edges = [16 * (tiles * c // nc) for c in range(nc + 1)]
                first = len(toks)
                toks.extend((int(tok_off[i]), int(q_starts[i])) for i in members)
                tasks.extend((int(slots[members[0]]), first, len(members), c, edges[c], edges[c + 1], 0, 0)
                             for c in range(nc))
                shared[members] = p
                nparts[members] = nc
        self._cascade_memo = (key, (shared, nparts, tasks, toks))
        return shared, nparts, tasks, toks

    def plan(self, slots, q_lens, q_starts, split: int | None = None, fine_tail: bool = True,
             q_heads: int | None = None, fixed_layout: bool = False) -> StepPlan:
        """Allocate blocks for a step and pack its metadata on the GPU.

        ``slots[i]`` gets ``q_lens[i]`` new tokens whose rows in the caller's
        q/k/v tensors start at ``q_starts[i]``.  Allocation happens in list
        order, like the reference's row loop (paged_kv_cache.py:110-111).
        Raises before any launch on an over-long sequence or an exhausted pool.
        ``split`` (a multiple of 16) overrides the unit size chosen for the
        step; ``fine_tail`` gives the shortest sequences smaller units
        (``seq_unit_sizes``).  With ``q_heads`` (the query head count of the
        attention calls) and a supported shape, sequences with at least
        ``PREFILL_MIN_TOKENS`` new tokens are attended by the tensor-core
        prefill kernel, in tiles of 128 query rows; the rest by the split-K
        kernel, and decode sequences that share leading blocks (imported
        prefixes) have those keys attended once per group of sequences by
        the cascade kernel (``_cascade_groups``).  ``fixed_layout`` keeps the
        device addresses and launch sizes the per-layer kernels see the same
        from one decode step of a batch to the next (room for one block-table
        patch per sequence, the unit capacity rounded up to 64), so that a
        captured CUDA graph of the layers stays valid: ``plan.layout_key``
        changes whenever they do not.
        """
        slots = np.asarray(slots, dtype=np.int64)
        q_lens = np.asarray(q_lens, dtype=np.int64)
        q_starts = np.asarray(q_starts, dtype=np.int64)
        if slots.size == 0:
            raise ValueError("a step needs at least one sequence")
        if (q_lens <= 0).any():
            raise ValueError("every sequence of a step needs at least one new token")
        if len(q_lens) != len(slots) or len(q_starts) != len(slots):
            raise ValueError("slots, q_lens and q_starts must have the same length")
        if (q_starts < 0).any():
            raise ValueError("q_starts must be non-negative")
        if slots.min() < 0 or slots.max() >= self.batch_size:
            raise IndexError(f"cache slot out of range [0, {self.batch_size})")
        if len(np.unique(slots)) != len(slots):
            raise ValueError("a slot may appear only once per step")
        ctx = self.pos_host[slots]
        over = ctx + q_lens > self.max_seq_len
        if over.any():
            i = int(np.argmax(over))
            raise AssertionError(
                f"slot {int(slots[i])}: {int(ctx[i])} + {int(q_lens[i])} tokens exceed max_seq_len {self.max_seq_len}")
        sl = slots.tolist()
        tabs = self.block_tables
        S = len(sl)
        # allocation in list order, as the reference's row loop (only the tables that must grow allocate)
        have = np.fromiter((len(tabs[s]._physical_blocks) for s in sl), np.int64, S)
        need = (ctx + q_lens + self.block_size - 1) // self.block_size
        for i in np.flatnonzero(need > have).tolist():
            tabs[sl[i]].ensure_capacity(int(ctx[i] + q_lens[i]))
            have[i] = len(tabs[sl[i]]._physical_blocks)
        # block-table patches: entries the device mirror lacks (all of a table whose epoch changed)
        epochs = np.fromiter((tabs[s].epoch for s in sl), np.int64, S)
        done = np.where(epochs != self._sync_epoch[slots], 0, self._sync_len[slots])
        patches = []
        for i in np.flatnonzero(have > done).tolist():
            s_, blocks = sl[i], tabs[sl[i]]._physical_blocks
            patches.extend((s_, lb, blocks[lb]) for lb in range(int(done[i]), int(have[i])))
        self._sync_epoch[slots] = epochs
        self._sync_len[slots] = have
        P = len(patches)
        T = int(q_lens.sum())
        # every query token is one work item attending over keys [0, ctx + i]
        kv = np.repeat(ctx + 1, q_lens) + (np.arange(T) - np.repeat(np.cumsum(q_lens) - q_lens, q_lens))
        routed = (q_lens >= self.PREFILL_MIN_TOKENS) if self.prefill_supported(q_heads) else np.zeros(S, bool)
        dec = ~routed
        if self.cascade_supported(q_heads) and dec.any():
            shared, nparts, ctasks, ctoks = self._cascade_groups(slots, q_lens, q_starts, ctx, dec,
                                                                 q_heads // self.n_heads, epochs)
        else:
            shared, nparts, ctasks, ctoks = np.zeros(S, np.int32), np.zeros(S, np.int32), [], []
        tok_dec = np.repeat(dec, q_lens)
        kv_dec = kv[tok_dec] - np.repeat(shared.astype(np.int64), q_lens)[tok_dec]  # each query's own keys
        if split is None:
            split = self.split_for(max(1, int(kv_dec.sum())))
        if split <= 0 or split % 16:
            raise ValueError(f"split ({split}) must be a positive multiple of 16")
        seq_keys = q_lens * (ctx + 1) + q_lens * (q_lens - 1) // 2 - q_lens * shared
        seq_split = np.zeros(S, dtype=np.int32)  # 0: the prefill kernel serves the sequence
        if dec.any():
            seq_split[dec] = (seq_unit_sizes(seq_keys[dec], split, self.decode_workers) if fine_tail else split)
            # a decode sequence with cascade parts whose own keys fit in one unit of modest size gets that one
            # unit: the decode kernel then merges the cascade parts in the unit's epilogue, and a step of such
            # sequences needs no end-of-launch merge (enough of them keep the SMs busy)
            one = dec & (shared > 0) & (q_lens == 1) & (seq_keys <= self.CASCADE_OWN_UNIT_MAX * split)
            if one.sum() * 2 >= self.decode_workers:
                seq_split[one] = (seq_keys[one] + 15) // 16 * 16
        item_split = np.repeat(seq_split.astype(np.int64), q_lens)
        n_units = int(((kv_dec + item_split[item_split > 0] - 1) // item_split[item_split > 0]).sum())
        n_casc = int(nparts.sum())  # partial slots of the cascade parts (q_len 1: one item per sequence)
        max_units = max(1, n_units + n_casc)
        if fixed_layout:
            max_units = (max_units + 63) // 64 * 64
        tiles = []
        if routed.any():
            tt = _lib.load().nf_prefill_tile_rows(self.head_dim) // (q_heads // self.n_heads)  # tokens per item
            for i in np.flatnonzero(routed).tolist():
                n, c, r0 = int(q_lens[i]), int(ctx[i]), int(q_starts[i])
                for t0 in reversed(range(0, n, tt)):  # most keys first
                    tiles.append((int(slots[i]), r0 + t0, min(tt, n - t0), c + t0))

        n_tiles = len(tiles)
        sched = _prefill_order(tiles, self.n_heads) if n_tiles else np.zeros(0, np.int32)
        # seqs, per-sequence unit sizes, block-table patches (room for one per sequence with fixed_layout),
        # prefill tiles and order, shared keys, cascade tasks and query records; the device outputs follow
        p_room = max(P, S) if fixed_layout else P
        off_tiles = _align4(S * 5 + p_room * 3)
        off_sched = off_tiles + 4 * n_tiles
        n_ct, n_tok = len(ctasks), len(ctoks)
        off_shared = _align4(off_sched + sched.size)
        off_ct = _align4(off_shared + 2 * S)
        off_tok = off_ct + 8 * n_ct
        host = np.zeros(off_tok + 2 * n_tok, dtype=np.int32)
        host[: S * 4] = np.stack([slots, q_starts, q_lens, ctx], axis=1).reshape(-1)
        host[S * 4: S * 5] = seq_split
        if P:
            host[S * 5: S * 5 + P * 3] = np.asarray(patches, dtype=np.int32).reshape(-1)
        if n_tiles:
            host[off_tiles:off_sched] = np.asarray(tiles, dtype=np.int32).reshape(-1)
            host[off_sched:off_sched + sched.size] = sched
        if n_ct:
            host[off_shared:off_shared + 2 * S] = np.stack([shared, nparts], axis=1).reshape(-1)
            host[off_ct:off_tok] = np.asarray(ctasks, dtype=np.int32).reshape(-1)
            host[off_tok:] = np.asarray(ctoks, dtype=np.int32).reshape(-1)
        off_slot = _align4(host.size)
        off_src = off_slot + T
        off_items = _align4(off_src + T)
        off_units = off_items + 4 * T
        off_counts = off_units + _lib.UNIT_FIELDS * max_units
        meta = self._meta.get(off_counts + 4)
        meta[: host.size].copy_(torch.from_numpy(host).pin_memory(), non_blocking=True)
        pos_dev = self._pos_buf.get(T)

        plan = StepPlan(slots, q_lens, q_starts, ctx, split, max_units, seq_split)
        plan.upload_bytes = host.nbytes
        # what a captured graph of the per-layer kernels depends on besides the cache's own buffers
        plan.layout_key = (meta.data_ptr(), off_ct, off_tok, off_slot, off_units, off_counts, max_units, S, T,
                           n_ct, n_tok, n_tiles, q_heads)
        plan.decode_units = n_units
        plan.q_heads = q_heads
        plan.shared_keys = shared
        plan.n_casc_tasks, plan.n_casc_toks = n_ct, n_tok
        plan.casc_tasks = meta[off_ct: off_tok]
        plan.casc_toks = meta[off_tok: off_tok + 2 * n_tok]
        plan.n_tiles = n_tiles
        plan.tiles = meta[off_tiles: off_tiles + 4 * n_tiles]
        plan.sched = meta[off_sched: off_sched + sched.size]
        plan.seqs = meta[: S * 4]
        plan.slot_mapping = meta[off_slot: off_slot + T]
        plan.src_rows = meta[off_src: off_src + T]
        plan.items = meta[off_items: off_items + 4 * T]
        plan.units = meta[off_units: off_units + _lib.UNIT_FIELDS * max_units]
        plan.counts = meta[off_counts: off_counts + 4]
        plan.positions = pos_dev[:T]
        lib = _lib.load()
        _lib.check(lib.nf_pack_step(
            meta.data_ptr(), S, meta.data_ptr() + 4 * S * 5 if P else None, P,
            self.bt_dev.data_ptr(), self.batch_size, self.max_blocks_per_seq, self.block_size,
            self.num_blocks, split, meta.data_ptr() + 4 * S * 4,
            meta.data_ptr() + 4 * off_shared if n_ct else None, plan.slot_mapping.data_ptr(), plan.src_rows.data_ptr(),
            plan.positions.data_ptr(), plan.items.data_ptr(), plan.units.data_ptr(), plan.counts.data_ptr(),
            T, max_units, self.status.data_ptr(), _lib.stream_handle(self.device)), "nf_pack_step")
        self._plan = plan
        return plan

    def _close(self, plan: StepPlan) -> None:
        self.pos_host[plan.slots] = plan.ctx_before + plan.q_lens
        self.steps_closed += 1
        plan.closed = True
        if self._plan is plan:
            self._plan = None

    # ------------------------------------------------------------------ per-layer kernels
    def append_step(self, layer_id: int, key: torch.Tensor, value: torch.Tensor, plan: StepPlan) -> None:
        """Scatter the step's new K/V rows (rows of ``key``/``value``: n_rows x H*D) into layer ``layer_id``."""
        if plan.closed:
            raise RuntimeError("step plan already closed")
        if not key.is_cuda:
            _lib.require_cuda(key, "key")
        w = self._row_width
        for name, t in (("key", key), ("value", value)):
            if t.dim() != 2 or t.shape[1] != w or t.stride(1) != 1:
                raise ValueError(f"{name} must be (rows, {w}) with unit column stride")
        if key.shape[0] < plan.rows_needed or value.shape[0] < plan.rows_needed:
            raise ValueError(f"key/value have {key.shape[0]} rows, the step uses rows up to {plan.rows_needed}")
        if not 0 <= layer_id < self.num_layers:
            raise IndexError(f"layer_id {layer_id} out of range [0, {self.num_layers})")
        last = layer_id == self.num_layers - 1
        a = plan.append_args
        if a is None:  # the plan's part of the call, the same for every layer
            a = plan.append_args = _lib.NfAppendArgs(
                pool_rows=self._pool_rows, pool_dtype=self._dt_code, n_tokens=plan.n_tokens,
                num_kv_heads=self.n_heads, head_dim=self.head_dim, n_seqs=plan.n_seqs,
                slot_mapping=plan.slot_mapping.data_ptr(), src_rows=plan.src_rows.data_ptr(),
                seqs=plan.seqs.data_ptr(), status=self._status_ptr)
        a.k_pool, a.v_pool = self._k_ptr[layer_id], self._v_ptr[layer_id]
        a.k_new, a.v_new = key.data_ptr(), value.data_ptr()
        a.k_src_row_stride, a.v_src_row_stride = key.stride(0), value.stride(0)
        a.src_dtype = _lib.dtype_code(key.dtype)
        a.pos_out = self._pos_ptr if last else None
        rc = _lib.load().nf_kv_append_args(ctypes.addressof(a), self._stream())
        if rc:
            _lib.check(rc, "nf_kv_append")
        if last:
            self._close(plan)

    def projection_fusable(self, x: torch.Tensor, plan: StepPlan, n_q: int) -> bool:
        """True when ``project_append_step`` serves this step: 16-bit pools and x of the same dtype, the step's
        rows laid out as its tokens in order (row t = token t), widths multiples of 64."""
        return (self.dtype in (torch.bfloat16, torch.float16) and x.dtype == self.dtype and x.dim() == 2
                and x.stride(1) == 1 and x.shape[0] == plan.n_tokens and plan.rows_needed == plan.n_tokens
                and bool((plan.q_starts == np.cumsum(plan.q_lens) - plan.q_lens).all())
                and n_q % 64 == 0 and (self.n_heads * self.head_dim) % 64 == 0 and x.shape[1] % 8 == 0)

    def project_append_step(self, layer_id: int, x: torch.Tensor, weight: torch.Tensor, bias, plan: StepPlan,
                            q_out: torch.Tensor) -> torch.Tensor:
        """The input projection fused with the KV append for layer ``layer_id``: ``[q | k | v] = x weight^T
        (+ bias)`` on the tensor cores, q into ``q_out`` (rows, n_q) and k/v straight into the pools
        (``nf_qkv_append``).  ``weight``: (n_q + 2 Hkv*D, in_features), the q, k and v weights stacked.
        Same plan bookkeeping as ``append_step`` (``pos`` advances after the last layer)."""
        if plan.closed:
            raise RuntimeError("step plan already closed")
        if not 0 <= layer_id < self.num_layers:
            raise IndexError(f"layer_id {layer_id} out of range [0, {self.num_layers})")
        n_kv = self.n_heads * self.head_dim
        n_q = q_out.shape[1]
        if weight.shape != (n_q + 2 * n_kv, x.shape[1]) or not weight.is_contiguous() or weight.dtype != self.dtype:
            raise ValueError(f"weight must be a contiguous ({n_q + 2 * n_kv}, {x.shape[1]}) {self.dtype} tensor")
        if not self.projection_fusable(x, plan, n_q) or q_out.stride(1) != 1 or q_out.dtype != self.dtype:
            raise ValueError("this step cannot use the fused projection (see projection_fusable)")
        last = layer_id == self.num_layers - 1
        lib = _lib.load()
        _lib.check(lib.nf_qkv_append(
            x.data_ptr(), x.stride(0), x.shape[0], weight.data_ptr(), bias.data_ptr() if bias is not None else None,
            x.shape[1], n_q, n_kv, q_out.data_ptr(), q_out.stride(0), self.k[layer_id].data_ptr(),
            self.v[layer_id].data_ptr(), self.num_blocks * self.block_size, _lib.dtype_code(self.dtype),
            plan.slot_mapping.data_ptr(), plan.seqs.data_ptr(), plan.n_seqs,
            self.pos.data_ptr() if last else None, self.status.data_ptr(), _lib.stream_handle(self.device)),
            "nf_qkv_append")
        if last:
            self._close(plan)
        return q_out

    def attention_step(self, layer_id: int, q: torch.Tensor, plan: StepPlan, out: torch.Tensor,
                       scale: float | None = None, events=None, exchange=None) -> torch.Tensor:
        """out[row] = attention of q[row] over the cached keys of its sequence, for the step's rows.

        ``q``/``out``: (rows, Hq*D) in the pool dtype with unit column stride.
        Rows not in the step are left untouched.  ``events``: optional three
        CUDA events recorded before the prefill launch, between the prefill and
        the split-K launches, and after them (kernel timing).  ``exchange``
        (a ``sharding.PeerExchange``, with ``out`` one of its ``out`` views):
        the kernels also store the rows into the other ranks' gathered
        buffers and the launch ends once every rank's rows are in this one's.
        """
        if not q.is_cuda:
            _lib.require_cuda(q, "q")
        D = self.head_dim
        if q.dim() != 2 or q.shape[1] % self._row_width != 0 or q.stride(1) != 1:
            raise ValueError(f"q must be (rows, Hq*{D}) with Hq a multiple of {self.n_heads}")
        if out.shape != q.shape or out.stride(1) != 1:
            raise ValueError("out must have q's shape")
        if q.dtype != self.dtype or out.dtype != self.dtype:
            raise ValueError(f"q/out dtype must be the cache dtype {self.dtype}")
        if q.shape[0] < plan.rows_needed:
            raise ValueError(f"q has {q.shape[0]} rows, the step uses rows up to {plan.rows_needed}")
        if not 0 <= layer_id < self.num_layers:
            raise IndexError(f"layer_id {layer_id} out of range [0, {self.num_layers})")
        hq = q.shape[1] // D
        if (plan.n_tiles or plan.n_casc_tasks) and hq != plan.q_heads:
            raise ValueError(f"the plan's prefill tiles / cascade groups are for {plan.q_heads} query heads, q has {hq}")
        if scale is None:
            scale = 1.0 / math.sqrt(D)
        lib = _lib.load()
        stream = self._stream()
        gather = exchange.next(out) if exchange is not None else None
        gref = ctypes.byref(gather) if gather is not None else None
        kp, vp = self._k_ptr[layer_id], self._v_ptr[layer_id]
        qp, op, qs, os_ = q.data_ptr(), out.data_ptr(), q.stride(0), out.stride(0)
        if events is not None:
            events[0].record()
        if plan.n_tiles:
            _lib.check(lib.nf_prefill_attention_gather(
                op, os_, qp, qs, min(q.shape[0], out.shape[0]), kp, vp, self._dt_code, hq, self.n_heads, D,
                self.block_size, self.num_blocks, self._bt_ptr, self.max_blocks_per_seq, plan.tiles.data_ptr(),
                plan.n_tiles, plan.sched.data_ptr(), self._pf_queue.data_ptr(), float(scale), gref,
                self._status_ptr, stream), "nf_prefill_attention")
        if events is not None:
            events[1].record()
        if plan.decode_units:
            max_items = plan.n_tokens
            if plan.ws_sizes is None or plan.ws_sizes[0] != hq:  # the same for every layer of the step
                pf, ci = _lib.workspace_sizes(plan.max_units, max_items, hq, self.n_heads, D, self.dtype)
                plan.ws_sizes = (hq, pf, ci)
                plan.decode_args = _lib.NfAttentionArgs(
                    dtype=self._dt_code, num_q_heads=hq, num_kv_heads=self.n_heads, head_dim=D,
                    block_size=self.block_size, num_blocks=self.num_blocks, block_tables=self._bt_ptr,
                    max_blocks_per_seq=self.max_blocks_per_seq, max_items=max_items, max_units=plan.max_units,
                    split_tokens=plan.split, items=plan.items.data_ptr(), units=plan.units.data_ptr(),
                    counts=plan.counts.data_ptr(), status=self._status_ptr)
            _, pf, ci = plan.ws_sizes
            ws = self._ws_partials.get(pf)
            cnt = self._ws_counters.get(ci)
            if plan.n_casc_tasks:
                # partials over the shared keys, merged by the decode launch with each query's own keys
                _lib.check(lib.nf_cascade_attention(
                    ws.data_ptr(), ws.numel(), qp, qs, q.shape[0], kp, vp, self._dt_code,
                    hq, self.n_heads, D, self.block_size, self.num_blocks, self._bt_ptr,
                    self.max_blocks_per_seq, plan.items.data_ptr(), plan.counts.data_ptr(), max_items,
                    plan.max_units, plan.casc_tasks.data_ptr(),
                    plan.n_casc_tasks, plan.casc_toks.data_ptr(), plan.n_casc_toks, float(scale),
                    self._status_ptr, stream), "nf_cascade_attention")
            a = plan.decode_args
            a.out, a.out_row_stride, a.q, a.q_row_stride, a.k_pool, a.v_pool = op, os_, qp, qs, kp, vp
            a.scale = scale
            a.ws_partials, a.ws_partial_floats = ws.data_ptr(), ws.numel()
            a.ws_counters, a.ws_counter_ints = cnt.data_ptr(), cnt.numel()
            a.gather = ctypes.addressof(gather) if gather is not None else None
            rc = lib.nf_paged_attention_args(ctypes.addressof(a), stream)
            if rc:
                _lib.check(rc, "nf_paged_attention")
        elif gather is not None:  # every row came from the prefill kernel: signal the peers on their own
            _lib.check(lib.nf_exchange_barrier(gref, self._status_ptr, stream), "nf_exchange_barrier")
        if events is not None:
            events[2].record()
        return out

    # ------------------------------------------------------------------ diagnostics
    def check_status(self) -> None:
        """Raise if any kernel flagged a problem (reads the device status word: synchronises)."""
        st = int(self.status.item())
        if st:
            self.status.zero_()
            raise _lib.NifreError(f"device status {st:#x} (bad block={st & 1}, unit overflow={st >> 1 & 1}, "
                                  f"wait timeout={st >> 2 & 1}, bad slot={st >> 3 & 1}, bad tile={st >> 4 & 1}, "
                                  f"bad shared keys={st >> 5 & 1})")

    def device_block_table(self, slot: int, n: int | None = None) -> list[int]:
        row = self.bt_dev[slot].tolist()
        return row[: len(self.block_tables[slot]) if n is None else n]


def _align4(n: int) -> int:
    return (n + 3) & ~3
