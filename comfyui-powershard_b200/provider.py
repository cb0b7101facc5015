"""The ``b200`` attention provider behind PowerShard's provider API.

``B200Provider()(q, k, v, options)`` has the calling convention of the
reference's provider adapters (``FlashProvider.__call__``,
powershard/attention_providers.py:101-116, invoked from
``AttentionDispatcher.__call__``, attention_policy.py:101-149):

* BLHD tensors ``q [B,Lq,Hq,D]``, ``k/v [B,Lk,Hk,D]`` (fp16 or bf16, CUDA,
  any strides with a contiguous head dim);
* returns a new tensor of q's dtype/device, shape ``[B,Lq,Hq,Dv]``;
* raises ``UnsupportedAttention`` BEFORE launching for anything the kernel
  does not compute (mask, causal, window, ALiBi, dropout, attention
  probabilities, head_dim != 128, other dtypes, CPU tensors), so the
  dispatcher may fall back (attention_policy.py:135-147);
* any failure after that point is a RuntimeError/ValueError and propagates.

``identity`` is the fingerprint the dispatcher compares against the probe's
record (attention_policy.py:97-99).
"""
from __future__ import annotations

import torch

from . import _lib, ops
from .contract import AttentionOptions, UnsupportedAttention, validate

NAME = "b200"


class B200Provider:
    name = NAME

    def __init__(self):
        _lib.load()
        self.identity = _lib.library_identity()
        self.identity["provider"] = NAME
        self._status = {}
        self._workspaces = {}

    def _status_for(self, device: torch.device) -> ops.DeviceStatus:
        key = device.index if device.index is not None else torch.cuda.current_device()
        if key not in self._status:
            self._status[key] = ops.DeviceStatus(torch.device("cuda", key))
        return self._status[key]

    def check(self, q, k, v, o: AttentionOptions):
        """Raise UnsupportedAttention for every request outside the kernel."""
        validate(q, k, v, o)
        if o.mask is not None:
            raise UnsupportedAttention("b200: arbitrary masks are not supported")
        if o.causal:
            raise UnsupportedAttention("b200: causal attention is not implemented (non-causal DiT kernel)")
        if o.window_size != (-1, -1) or o.alibi_slopes is not None:
            raise UnsupportedAttention("b200: window/ALiBi are not supported")
        if o.dropout_p:
            raise UnsupportedAttention("b200: dropout is not supported")
        if o.return_attn_probs:
            raise UnsupportedAttention("b200: attention probabilities/LSE are not returned")
        if q.shape[-1] != 128 or v.shape[-1] != 128:
            raise UnsupportedAttention("b200: head_dim 128 only")
        if q.dtype not in (torch.float16, torch.bfloat16):
            raise UnsupportedAttention("b200: fp16/bf16 inputs required")
        _lib.require_cuda(q, "b200")

    def __call__(self, q, k, v, o: AttentionOptions | None = None):
        o = o or AttentionOptions()
        self.check(q, k, v, o)
        status = self._status_for(q.device)
        status.poll()
        q, k, v = (x if _tma_ok(x) else x.contiguous() for x in (q, k, v))
        scale = q.shape[-1] ** -0.5 if o.softmax_scale is None else float(o.softmax_scale)
        out = torch.empty(q.shape[:-1] + (v.shape[-1],), dtype=q.dtype, device=q.device)
        with torch.cuda.device(q.device):
            ops.attention_blhd(q, k, v, out, scale, status, self._workspace_for(q.device))
        return out

    def _workspace_for(self, device):
        """Attention scratch per (device, current stream)."""
        key = (device.index, torch.cuda.current_stream(device).cuda_stream)
        ws = self._workspaces.get(key)
        if ws is None:
            ws = self._workspaces[key] = ops.attention_workspace(device)
        return ws


def _tma_ok(t: torch.Tensor) -> bool:
    """Strides the TMA maps accept without a copy: unit head-dim stride,
    others multiples of 8 elements (16 bytes), 16-byte aligned base."""
    return (t.stride(3) == 1 and all(s % 8 == 0 for s in t.stride()[:3])
            and t.data_ptr() % 16 == 0)
