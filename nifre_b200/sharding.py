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
