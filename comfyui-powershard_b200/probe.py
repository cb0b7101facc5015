"""Numerical certification probe of the b200 provider.

The counterpart of powershard/attention_probe.py:6-53 for ``provider ==
"b200"``: the same seeded geometry (batch 2, non-contiguous q via a
stride-2 head dim, lengths 5/7, scales .13/.37), checked in fp16 (the
reference probe dtype) and bf16 (the Ulysses wire dtype) against an fp32
softmax(QK^T)V computed by torch on the same device, atol = rtol = 7e-3 for
fp16 and 2e-2 for bf16.  The reference's causal case (7, 7, .2) must raise
UnsupportedAttention, since this provider is non-causal by design.

Run as ``python -m powershard_b200.probe [head_dim] [heads]``; prints one
JSON line like the reference probe.
"""
from __future__ import annotations

import json
import sys

import torch

from .contract import AttentionOptions, UnsupportedAttention


def _fp32_attention(q, k, v, scale):
    qf, kf, vf = (x.float().transpose(1, 2) for x in (q, k, v))
    p = torch.softmax((qf @ kf.transpose(-1, -2)) * scale, dim=-1)
    return (p @ vf).transpose(1, 2)


def probe(head_dim: int = 128, heads: int = 4, device: str = "cuda:0"):
    from .provider import B200Provider
    provider = B200Provider()
    generator = torch.Generator(device=device).manual_seed(1729)
    checks = []
    for dtype, tol in ((torch.float16, 7e-3), (torch.bfloat16, 2e-2)):
        for lq, lk, scale in ((5, 7, .13), (5, 7, .37)):
            q = torch.randn((2, lq, heads, head_dim * 2), device=device, dtype=dtype, generator=generator)[..., ::2]
            k = torch.randn((2, lk, heads, head_dim), device=device, dtype=dtype, generator=generator)
            v = torch.randn((2, lk, heads, head_dim), device=device, dtype=dtype, generator=generator)
            o = AttentionOptions(softmax_scale=scale)
            ref = _fp32_attention(q, k, v, scale)
            for _ in range(2):
                actual = provider(q, k, v, o)
            torch.cuda.synchronize(device)
            if not torch.isfinite(actual).all():
                raise FloatingPointError("probe produced NaN/Inf")
            torch.testing.assert_close(actual.float(), ref, atol=tol, rtol=tol)
            checks.append(dict(dtype=str(dtype), lq=lq, lk=lk, scale=scale,
                               max_abs=(actual.float() - ref).abs().max().item()))
    q = torch.randn((2, 7, heads, head_dim), device=device, dtype=torch.float16, generator=generator)
    try:
        provider(q, q, q, AttentionOptions(softmax_scale=.2, causal=True))
        causal = "computed"
    except UnsupportedAttention:
        causal = "UnsupportedAttention"
    if causal != "UnsupportedAttention":
        raise AssertionError("causal request must raise UnsupportedAttention")
    return dict(status="PASS", import_result="PASS", kernel_result="PASS", numerical_result="PASS",
                identity=provider.identity,
                geometry=dict(head_dim=head_dim, heads=heads, dtype="bfloat16", layout="BLHD",
                              kv_heads=heads, gqa_certified=False),
                torch=str(torch.__version__), device=torch.cuda.get_device_name(device),
                checks=checks, causal=causal)


if __name__ == "__main__":
    try:
        result = probe(int(sys.argv[1]) if len(sys.argv) > 1 else 128,
                       int(sys.argv[2]) if len(sys.argv) > 2 else 4)
    except Exception as error:  # the process ends; a broken context is never reused
        result = dict(status="FAIL", reason=f"{type(error).__name__}: {error}")
    print(json.dumps(result))
