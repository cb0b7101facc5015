"""The provider contract of PowerShard's attention API.

When PowerShard itself is importable (the package runs inside a ComfyUI
install next to ComfyUI-PowerShard), its own ``UnsupportedAttention``,
``AttentionOptions`` and ``validate`` are re-exported, so the reference
``AttentionDispatcher`` catches this provider's UnsupportedAttention and falls
back exactly as it does for its other providers
(powershard/attention_policy.py:135-147).  Otherwise this module defines the
same three names with the same semantics:

* ``UnsupportedAttention`` - a RuntimeError raised BEFORE any kernel launch
  for a request the provider does not cover (attention_contract.py:14-15);
* ``AttentionOptions`` - frozen option record (attention_contract.py:18-29);
* ``validate(q, k, v, o)`` - BLHD shape/dtype/option checks returning
  (b, lq, hq, d, lk, hk, dv) (attention_contract.py:32-56).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

try:  # running next to ComfyUI-PowerShard: share its exception and option types
    from powershard.attention_contract import (  # type: ignore
        AttentionOptions, UnsupportedAttention, validate)
    SHARED_WITH_POWERSHARD = True
except ImportError:  # standalone: same names, same behaviour
    SHARED_WITH_POWERSHARD = False

    class UnsupportedAttention(RuntimeError):
        """Predictable absence of a semantic, raised before any CUDA kernel runs."""

    @dataclass(frozen=True)
    class AttentionOptions:
        softmax_scale: float | None = None
        mask: object = None
        causal: bool = False
        causal_alignment: str = "upper_left"
        dropout_p: float = 0.0
        window_size: tuple = (-1, -1)
        alibi_slopes: object = None
        deterministic: bool = False
        return_attn_probs: bool = False
        layout: str = "BLHD"

    def validate(q, k, v, o):
        """BLHD Q [B,Lq,Hq,D], K/V [B,Lk,Hk,D(v)]; raises ValueError on misuse."""
        if o.layout != "BLHD" or any(x.ndim != 4 for x in (q, k, v)):
            raise ValueError("explicit BLHD layout requires four Q/K/V axes")
        b, lq, hq, d = q.shape
        bk, lk, hk, dk = k.shape
        bv, lv, hv, dv = v.shape
        if (b != bk or b != bv or lk != lv or hk != hv or d != dk
                or not min(b, hq, hk, d, dv, lk) or hq % hk):
            raise ValueError("incompatible Q/K/V: batch, K/V length, heads, Q/K dim or GQA")
        if (len({x.device for x in (q, k, v)}) != 1 or len({x.dtype for x in (q, k, v)}) != 1
                or not q.is_floating_point()):
            raise ValueError("Q/K/V must share one floating dtype and device")
        if not 0 <= o.dropout_p < 1 or o.causal_alignment not in ("upper_left", "bottom_right"):
            raise ValueError("invalid dropout or causal_alignment")
        if len(o.window_size) != 2 or any(not isinstance(x, int) or x < -1 for x in o.window_size):
            raise ValueError("window_size: two integers >= -1")
        if o.softmax_scale is not None and not math.isfinite(o.softmax_scale):
            raise ValueError("softmax_scale must be finite")
        if o.mask is not None:
            if o.mask.device != q.device or (o.mask.dtype != torch.bool and not o.mask.is_floating_point()):
                raise ValueError("mask: bool/floating on the same device")
            if torch.broadcast_shapes(o.mask.shape, (b, hq, lq, lk)) != (b, hq, lq, lk):
                raise ValueError("mask is not broadcastable to B,H,Lq,Lk")
        if o.alibi_slopes is not None:
            if o.alibi_slopes.shape not in ((hq,), (b, hq)) or o.alibi_slopes.device != q.device:
                raise ValueError("ALiBi slopes: [Hq] or [B,Hq] on the same device")
        return b, lq, hq, d, lk, hk, dv

__all__ = ["AttentionOptions", "UnsupportedAttention", "validate", "SHARED_WITH_POWERSHARD"]
