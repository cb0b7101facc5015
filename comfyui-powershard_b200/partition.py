"""Token / head partition of the Ulysses exchange.

``shard_bounds`` follows powershard/config.py:107-112 (ceil-width contiguous
token shards, the last ranks may be empty); ``UlyssesGeometry`` collects the
per-rank sizes the reference derives in ulysses_to_sequence
(powershard/wan_model.py:343-364): width = ceil(L/W) token rows per source
segment and h = ceil(H/W) head slots per rank, H zero-padded to h*W.

Image models split their image segment differently: ``split_sizes`` and
``ImageLayout`` follow powershard/image_layout.py:12-36 (balanced parts, the
first n % W ranks one row longer).  A geometry built with ``sizes`` uses that
split; its width is max(sizes), the layout's ``chunk``.
"""
from __future__ import annotations

import math
from dataclasses import dataclass


def split_sizes(n: int, world: int) -> list[int]:
    """Rows of each rank when n rows are split over `world` ranks, the first
    n % world ranks one row longer (powershard/image_layout.py:12-15)."""
    base, extra = divmod(int(n), int(world))
    return [base + (1 if r < extra else 0) for r in range(int(world))]


class ImageLayout:
    """Sequence layout of an image-model block: consecutive segments
    [(rows, split)], exactly one split across ranks (the image tokens), the
    rest replicated on every rank (powershard/image_layout.py:18-36).  Only
    the attributes the attention override reads are kept: total, world,
    rank, split_start, split_len, sizes, a, b, local_len, chunk."""

    def __init__(self, segments, world: int, rank: int):
        self.segments = [(int(n), bool(s)) for n, s in segments]
        if sum(1 for _, s in self.segments if s) != 1:
            raise ValueError(f"exactly one split segment required: {segments}")
        self.world, self.rank = int(world), int(rank)
        self.total = sum(n for n, _ in self.segments)
        start = 0
        for n, s in self.segments:
            if s:
                self.split_start, self.split_len = start, n
            start += n
        self.sizes = split_sizes(self.split_len, self.world)
        self.a = self.split_start + sum(self.sizes[:self.rank])
        self.b = self.a + self.sizes[self.rank]
        self.local_len = self.total - self.split_len + (self.b - self.a)
        self.chunk = max(self.sizes) if self.sizes else 0


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
    sizes: tuple | None = None  # rows of each rank (balanced split); None: shard_bounds

    def __post_init__(self):
        if self.sizes is not None:
            sizes = tuple(int(x) for x in self.sizes)
            if len(sizes) != self.world or min(sizes) < 0 or sum(sizes) != self.total:
                raise ValueError(f"sizes {sizes} do not split {self.total} rows over {self.world} ranks")
            object.__setattr__(self, "sizes", sizes)

    @property
    def width(self) -> int:
        """Token rows per source segment of the exchange: ceil(L/W), or the
        longest part of a balanced split."""
        if self.sizes is not None:
            return max(self.sizes)
        return math.ceil(self.total / self.world)

    def seg_valid(self) -> list[int]:
        """Valid rows of each source segment of the receive buffer."""
        if self.sizes is not None:
            return list(self.sizes)
        w = self.width
        return [max(0, min(w, self.total - s * w)) for s in range(self.world)]


    @property
    def heads_per_rank(self) -> int:
        """Head slots per rank, ceil(H/W)."""
        return math.ceil(self.heads / self.world)

    @property
    def padded_heads(self) -> int:
        return self.heads_per_rank * self.world

    @property
    def bounds(self):
        if self.sizes is not None:
            a = sum(self.sizes[:self.rank])
            return a, a + self.sizes[self.rank]
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

    def send_shape(self, batch: int | None = None):
        """[W, 3, width, h, D], or with a batch axis [W, 3, B, width, h, D]
        (the reference's packing, powershard/wan_model.py:356-361)."""
        if batch is None:
            return (self.world, 3, self.width, self.heads_per_rank, self.head_dim)
        return (self.world, 3, int(batch), self.width, self.heads_per_rank, self.head_dim)

    def out_shape(self, batch: int | None = None):
        """[W, width, h, D], or [W, B, width, h, D] (wan_model.py:373-376)."""
        if batch is None:
            return (self.world, self.width, self.heads_per_rank, self.head_dim)
        return (self.world, int(batch), self.width, self.heads_per_rank, self.head_dim)

    def exchanged_bytes(self, element_size: int, batch: int = 1) -> tuple[int, int]:
        """Bytes of the QKV send buffer and of the output send buffer of one
        call (the reference's send.numel() * element_size, wan_model.py:364, 381)."""
        n = 1
        for s in self.send_shape(batch):
            n *= s
        m = 1
        for s in self.out_shape(batch):
            m *= s
        return n * element_size, m * element_size
