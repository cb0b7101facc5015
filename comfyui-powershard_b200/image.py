"""Sequence-parallel attention override for image models (Flux double/single blocks).

Drop-in for powershard/image_parallel.py:67-110 (``SequenceAttention``), the
``optimized_attention_override`` that ``flux_double`` / ``flux_single``
(:162-206) put into a block's transformer_options.  The reference keeps the
queries local and all-gathers keys and values of the split image segment
(``assemble_full``, :45-52), so every rank computes attention over the whole
sequence for its local rows.  This override computes the same rows with the
Ulysses exchange instead: the image rows of q/k/v cross one all-to-all (each
rank then holds every image row for H/W heads), the text rows that every
rank already holds are taken locally, the joint attention kernel runs
[text; image] keys for this rank's heads, and the outputs return by an
all-to-all (image rows) and an all-gather over heads (text rows).

Same calling convention as the reference: ``override(func, q, k, v, heads,
*rest, skip_reshape=..., **kwargs)`` with q/k/v in the block's local layout
(``[B, H, local_len, D]`` when skip_reshape, else ``[B, local_len, H*D]``),
returning ``[B, local_len, H*D]`` (``[B, H, local_len, D]`` with
skip_output_reshape), the attention dtype of q.  The result is
softmax(Q K^T / sqrt(D)) V, the attention ComfyUI's optimized_attention
computes; `func` is not called on this path.

Cases outside the kernel's contract (an attention mask, keys appended inside
the attention, a replicated segment after the image segment, dtype or
head_dim the kernel does not take, CPU tensors) go to ``fallback`` - e.g. the
reference's own ``SequenceAttention(layout, stats)`` - when one is given, and
raise ``UnsupportedAttention`` otherwise, before anything is launched.
"""
from __future__ import annotations

import torch

from . import ops
from .contract import UnsupportedAttention
from .partition import ImageLayout, split_sizes  # noqa: F401  (re-exported for callers building layouts)
from .ulysses import UlyssesAttention

OVERRIDE_KEY = "optimized_attention_override"


def _mask_of(rest, kwargs):
    if rest and rest[0] is not None:
        return rest[0]
    return kwargs.get("mask")


class SequenceAttention:
    """``optimized_attention_override`` with the Ulysses exchange.

    layout: the block's image layout (``powershard.image_layout.Layout`` or
    ``ImageLayout``: total, world, rank, split_start, split_len, sizes,
    local_len); stats: the dict whose ``attention_calls`` counter the
    reference increments; engine: the ``UlyssesAttention`` of the sequence
    group (default: the default process group); fallback: callable with the
    override's signature for unsupported cases.
    """

    def __init__(self, layout, stats, engine: UlyssesAttention | None = None, fallback=None):
        self.layout, self.stats = layout, stats
        self.engine = engine if engine is not None else UlyssesAttention()
        self.fallback = fallback

    def _reason(self, q, k, v, heads, rest, kwargs, dim):
        lay = self.layout
        if _mask_of(rest, kwargs) is not None:
            return "attention mask"
        if k.shape[dim] != lay.local_len or v.shape[dim] != lay.local_len:
            return "keys appended inside the attention"
        if lay.split_start + lay.split_len != lay.total:
            return "replicated segment after the image segment"
        for t in (q, k, v):
            if t.device.type != "cuda" and self.engine.kernels is ops:
                return "CPU tensors"
            if t.dtype not in (torch.bfloat16, torch.float16) or t.dtype != q.dtype:
                return f"dtype {t.dtype}"
        width = q.shape[-1] if kwargs.get("skip_reshape", False) else q.shape[-1] // heads
        if width != 128 or (not kwargs.get("skip_reshape", False) and q.shape[-1] != heads * 128):
            return f"head_dim {width}"
        return None

    @staticmethod
    def _rows(t, b, heads, skip):
        """Batch row b as an [L, H, D] view (no copy)."""
        if skip:
            return t[b].transpose(0, 1)
        return t[b].unflatten(-1, (heads, t.shape[-1] // heads))

    def __call__(self, func, *args, **kwargs):
        q, k, v, heads = args[:4]
        rest = list(args[4:])
        skip = kwargs.get("skip_reshape", False)
        dim = 2 if skip else 1
        lay = self.layout
        if q.shape[dim] != lay.local_len:
            raise ValueError(f"sequence parallel: {q.shape[dim]} queries instead of {lay.local_len}")
        world, rank = self.engine.world_rank()
        if (world, rank) != (lay.world, lay.rank):
            raise ValueError(f"layout is for rank {lay.rank} of {lay.world}, group is rank {rank} of {world}")
        reason = self._reason(q, k, v, heads, rest, kwargs, dim)
        if reason is not None:
            if self.fallback is not None:
                return self.fallback(func, *args, **kwargs)
            raise UnsupportedAttention(f"B200 sequence attention: {reason}")
        self.stats["attention_calls"] = self.stats.get("attention_calls", 0) + 1

        batch, length, head_dim = q.shape[0], lay.local_len, 128
        prefix = lay.split_start
        out = torch.empty((batch, length, heads, head_dim), dtype=q.dtype, device=q.device)
        if world == 1 and self.engine.kernels is ops:
            # One rank holds the whole sequence: attend the caller's tensors in
            # place (strided TMA maps), no packing.
            from .provider import _tma_ok
            qv, kv, vv = (t.transpose(1, 2) if skip else t.unflatten(-1, (heads, head_dim)) for t in (q, k, v))
            qv, kv, vv = (t if _tma_ok(t) else t.contiguous() for t in (qv, kv, vv))
            with torch.cuda.device(q.device):
                status = self.engine._device_status(q.device)
                status.poll()
                ops.attention_blhd(qv, kv, vv, out, head_dim ** -0.5, status,
                                   self.engine._ws(q.device).get("workspace"))
            return out.permute(0, 2, 1, 3) if kwargs.get("skip_output_reshape", False) else \
                out.view(batch, length, heads * head_dim)
        for b in range(batch):
            qb, kb, vb = (self._rows(t, b, heads, skip) for t in (q, k, v))
            self.engine.forward_joint(
                (qb[:prefix], kb[:prefix], vb[:prefix]), (qb[prefix:], kb[prefix:], vb[prefix:]),
                total_img=lay.split_len, heads=heads, norm=ops.NORM_NONE, sizes=list(lay.sizes),
                out=(out[b, :prefix], out[b, prefix:]))
        if kwargs.get("skip_output_reshape", False):
            return out.permute(0, 2, 1, 3)
        return out.view(batch, length, heads * head_dim)


def options(transformer_options, layout, stats, engine: UlyssesAttention | None = None, fallback=None):
    """transformer_options with this override installed (powershard/image_parallel.py:113-116)."""
    opts = dict(transformer_options or {})
    opts[OVERRIDE_KEY] = SequenceAttention(layout, stats, engine, fallback)
    return opts
