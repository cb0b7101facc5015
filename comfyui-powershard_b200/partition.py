"""Token / head partition of the Ulysses exchange.

``shard_bounds`` follows powershard/config.py:107-112 (ceil-width contiguous
token shards, the last ranks may be empty); ``UlyssesGeometry`` collects the
per-rank sizes the reference derives in ulysses_to_sequence
(powershard/wan_model.py:343-364): width = ceil(L/W) token rows per source
segment and h = ceil(H/W) head slots per rank, H zero-padded to h*W.
"""
from __future__ import annotations

import math
from dataclasses import dataclass


def shard_bounds(rows: int, rank: int, world_size: int):
    """Rows [a, b) of `rank` under ceil-width sharding (torch.chunk semantics)."""
    if rows < 0 or world_size < 1 or not 0 <= rank < world_size:
        raise ValueError("invalid shard bounds")
    width = (rows + world_size - 1) // world_size
    return min(rows, rank * width), min(rows, (rank + 1) * width)


@dataclass(frozen=True)
class UlyssesGeometry:
    total: int          # L: tokens of the whole sequence
    heads: int          # H: attention heads of the layer
    head_dim: int       # D
    world: int          # W: ranks of the sequence-parallel group
    rank: int

    @property
    def width(self) -> int:
        """Token rows per source segment of the exchange, ceil(L/W)."""
        return math.ceil(self.total / self.world)

    @property
    def heads_per_rank(self) -> int:
        """Head slots per rank, ceil(H/W)."""
        return math.ceil(self.heads / self.world)

    @property
    def padded_heads(self) -> int:
        return self.heads_per_rank * self.world

    @property
    def bounds(self):
        return shard_bounds(self.total, self.rank, self.world)

    @property
    def n_local(self) -> int:
        a, b = self.bounds
        return b - a

    @property
    def heads_valid(self) -> int:
        """Real (non-padding) heads among this rank's head slots."""
        h = self.heads_per_rank
        return max(0, min(h, self.heads - self.rank * h))

    @classmethod
    def replicated(cls, rows: int, heads: int, head_dim: int, world: int) -> "UlyssesGeometry":
        """Geometry that packs `rows` tokens held by every rank (Flux text) for
        all W head blocks: rank 0 of a rows*W sequence has exactly those rows."""
        return cls(total=rows * world, heads=heads, head_dim=head_dim, world=world, rank=0)

    def send_shape(self):
        return (self.world, 3, self.width, self.heads_per_rank, self.head_dim)

    def out_shape(self):
        return (self.world, self.width, self.heads_per_rank, self.head_dim)

    def exchanged_bytes(self, element_size: int) -> tuple[int, int]:
        """Bytes of the QKV send buffer and of the output send buffer."""
        n = 1
        for s in self.send_shape():
            n *= s
        m = 1
        for s in self.out_shape():
            m *= s
        return n * element_size, m * element_size
