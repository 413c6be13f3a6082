"""KV-head sharding of the attention path over N GPUs (one process per GPU).

Attention is independent per KV head, so rank r of N owns KV heads
[r*Hkv/N, (r+1)*Hkv/N) and the matching query heads [r*Hq/N, (r+1)*Hq/N)
(a grouped-query group never straddles ranks).  Every rank keeps the same
block tables, positions and schedule (the host scheduler is deterministic),
appends and attends on its own pools, and the only exchange is one
all-gather per layer of the attention output, re-interleaved from
rank-major to head-major columns.  The reference runs on one device; this
is the multi-GPU form of the same computation.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class HeadShard:
    world: int
    rank: int
    num_q_heads: int
    num_kv_heads: int
    head_dim: int

    def __post_init__(self):
        if self.world <= 0 or not 0 <= self.rank < self.world:
            raise ValueError(f"rank {self.rank} out of range for world size {self.world}")
        if self.num_kv_heads % self.world:
            raise ValueError(f"{self.world} ranks must divide {self.num_kv_heads} KV heads")
        if self.num_q_heads % self.num_kv_heads:
            raise ValueError("num_q_heads must be a multiple of num_kv_heads")

    @property
    def kv_heads(self) -> int:
        return self.num_kv_heads // self.world

    @property
    def q_heads(self) -> int:
        return self.num_q_heads // self.world

    def q_columns(self) -> slice:
        w = self.q_heads * self.head_dim
        return slice(self.rank * w, (self.rank + 1) * w)

    def kv_columns(self) -> slice:
        w = self.kv_heads * self.head_dim
        return slice(self.rank * w, (self.rank + 1) * w)

    def local(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor):
        """This rank's columns of full (rows, H*D) projections."""
        return q[:, self.q_columns()], k[:, self.kv_columns()], v[:, self.kv_columns()]

    def gather(self, out_local: torch.Tensor, group=None, buffer: torch.Tensor | None = None) -> torch.Tensor:
        """All-gather the per-rank (rows, Hq/N*D) outputs into (rows, Hq*D), heads in global order."""
        import torch.distributed as dist

        rows, width = out_local.shape
        if buffer is None:
            buffer = torch.empty(self.world * rows, width, device=out_local.device, dtype=out_local.dtype)
        dist.all_gather_into_tensor(buffer, out_local.contiguous(), group=group)
        return buffer.view(self.world, rows, width).permute(1, 0, 2).reshape(rows, self.world * width)


class PeerExchange:
    """The gathered attention output of a KV-head shard, exchanged by the attention kernels themselves.

    Every rank holds ``slots`` gathered buffers of ``(max_rows, world * Hq/N * D)``
    (one per layer that may be in flight, so that a rank running ahead never
    overwrites a buffer a peer still reads) and a flag array of ``world``
    int32.  The buffers and flags are mapped into every other rank's process
    (CUDA IPC over NVLink); the attention kernels then store each output row
    into every rank's buffer at this rank's columns and end with a
    signal-and-wait on the flags (``nf_paged_attention_gather``), which
    replaces the attention launch + NCCL all-gather of ``HeadShard.gather``.
    All ranks must create the exchange and call ``next`` in the same order.
    The handles are swapped with one ``all_gather_object`` of the process
    group at construction; nothing else goes through the group.
    """

    def __init__(self, shard: HeadShard, max_rows: int, dtype: torch.dtype, device, slots: int = 1, group=None):
        import ctypes

        import torch.distributed as dist

        from nifre_b200 import _lib

        if shard.world > _lib.MAX_RANKS:
            raise ValueError(f"at most {_lib.MAX_RANKS} ranks in one exchange")
        self.shard = shard
        self.max_rows = max_rows
        self.width = shard.world * shard.q_heads * shard.head_dim
        self.buffers = torch.zeros(slots, max_rows, self.width, dtype=dtype, device=device)
        self.flags = torch.zeros(shard.world, dtype=torch.int32, device=device)
        # the exchange number, kept on the device: the signalling launch advances it, so that a CUDA graph of
        # exchanging launches replays with fresh epochs
        self.epoch_dev = torch.zeros(1, dtype=torch.int32, device=device)
        torch.cuda.synchronize(device)
        lib = _lib.load()
        mine = []
        for t in (self.buffers, self.flags):
            h = ctypes.create_string_buffer(64)
            off = ctypes.c_int64(0)
            _lib.check(lib.nf_ipc_handle(t.data_ptr(), h, ctypes.byref(off)), "nf_ipc_handle")
            mine.append((h.raw, off.value))
        every = [None] * shard.world
        dist.all_gather_object(every, mine, group=group)
        self._opened = []
        self.peer_bufs, self.peer_flags = [], []
        for r in range(shard.world):
            if r == shard.rank:
                self.peer_flags.append(self.flags.data_ptr())
                continue
            ptrs = []
            for raw, off in every[r]:
                p = ctypes.c_void_p()
                _lib.check(lib.nf_ipc_open(raw, off, ctypes.byref(p)), "nf_ipc_open")
                self._opened.append((p.value, off))
                ptrs.append(p.value)
            self.peer_bufs.append(ptrs[0])
            self.peer_flags.append(ptrs[1])
        self.epoch = 0
        dist.barrier(group=group)

    @staticmethod
    def slot_for(layer: int, step: int, layers: int) -> int:
        """Buffer of a layer's output in a step: two sets of one buffer per layer, alternating by step.

        A rank writes a peer's buffer for (step, layer) only after every rank
        has finished (step - 1, last layer), so with two sets a buffer is
        rewritten only once each rank has finished the step after the one it
        was read in."""
        return (step % 2) * layers + layer

    def out(self, slot: int, rows: int) -> torch.Tensor:
        """This rank's columns of gathered buffer ``slot``: a (rows, Hq/N*D) view with the gathered row stride."""
        return self.buffers[slot, :rows, self.shard.q_columns()]

    def gathered(self, slot: int, rows: int) -> torch.Tensor:
        """The whole gathered output of buffer ``slot``: (rows, Hq*D), heads in global order."""
        return self.buffers[slot, :rows]

    def next(self, out: torch.Tensor):
        """The NfGather of the next exchange, whose rows go to ``out`` (a view given by ``out``)."""
        from nifre_b200 import _lib

        off = out.data_ptr() - self.buffers.data_ptr()
        if not 0 <= off < self.buffers.numel() * self.buffers.element_size():
            raise ValueError("out must be a view of this exchange's gathered buffers")
        self.epoch += 1
        g = _lib.NfGather()
        g.n_ranks, g.rank, g.epoch = self.shard.world, self.shard.rank, self.epoch
        for i, base in enumerate(self.peer_bufs):
            g.peer_out[i] = base + off
        for r, f in enumerate(self.peer_flags):
            g.flags[r] = f
        g.epoch_counter = self.epoch_dev.data_ptr()
        return g

    def close(self) -> None:
        from nifre_b200 import _lib
        lib = _lib.load()
        for p, off in self._opened:
            lib.nf_ipc_close(p, off)
        self._opened = []
