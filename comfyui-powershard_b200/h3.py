"""H3 (MiniMax DiT) attention on the b200 kernels.

``attention_forward(self, x, rope_freqs=None, transformer_options=None)``
replaces powershard/attention.py:106-181 (installed by ``install_attention``,
:184-195, as ``module.forward``).  Same module attributes: ``qkv_proj``,
``q_norm`` / ``k_norm`` (RMSNorm over head_dim, weight [head_dim]),
``out_proj``, ``heads``, ``head_dim`` and the shared sequence state
``_ps_sequence`` (``enabled``, ``ulysses``, ``total`` and the counters).

The layout is LHD ([tokens, heads, head_dim], no batch axis).  q/k/v stay
strided views of the fused projection; one pre-pass kernel applies the
per-head RMSNorm and the split-half partial RoPE (rope_split_half,
attention.py:98-103: pairs (j, j + R/2) over the first R dims) and packs for
the exchange; then Ulysses (``ulysses`` true) or token mode, as the state
says.  The bf16 wire replaces the reference's fp16 scaled wire, so there is
no V scale all-reduce.
"""
from __future__ import annotations

import types

import torch

from . import ops
from .ulysses import UlyssesAttention

WIRE_DTYPE = torch.bfloat16


def _engine(module) -> UlyssesAttention:
    engine = getattr(module, "_ps_b200_engine", None)
    if engine is None:
        engine = UlyssesAttention(getattr(module, "_ps_b200_group", None))
        module._ps_b200_engine = engine
    return engine


def _identity_table(n: int, pairs: int, device) -> torch.Tensor:
    t = torch.zeros(n, pairs, 2, 2, dtype=torch.float32, device=device)
    t[..., 0, 0] = 1.0
    t[..., 1, 1] = 1.0
    return t


def attention_forward(self, x, rope_freqs=None, transformer_options=None):
    """x [n, dim] -> [n, dim] (local tokens of this rank)."""
    n = x.shape[0]
    heads, dim = self.heads, self.head_dim
    state = getattr(self, "_ps_sequence", None)
    sequence = state is not None and state.get("enabled", False)
    qkv = self.qkv_proj(x)
    if qkv.dtype != WIRE_DTYPE:
        qkv = qkv.to(WIRE_DTYPE)
    q, k, v = (t.view(n, heads, dim) for t in qkv.split(heads * dim, dim=-1))  # strided row views
    w_q, w_k = self.q_norm.weight, self.k_norm.weight
    if w_q.dtype not in (torch.float32, WIRE_DTYPE):
        w_q, w_k = w_q.float(), w_k.float()
    eps = getattr(self.q_norm, "eps", None) or 1e-6
    if rope_freqs is not None:
        table = rope_freqs[0, :, 0]
        pairs = table.shape[-3]
        if table.dtype != torch.float32 or table.stride()[1:] != (4, 2, 1) or table.data_ptr() % 16:
            table = table.float().contiguous()
    else:  # no RoPE: identity rotation of the first 8 pairs, the rest passes through
        pairs = 8
        table = _identity_table(n, pairs, x.device)
    engine = _engine(self)
    total = state["total"] if sequence else n
    kw = dict(total=total, heads=heads, eps=eps, norm_rope=ops.NORM_PER_HEAD, rope_split_pairs=pairs,
              state=state if sequence else None)
    if sequence and not state.get("ulysses", True):
        out = engine.forward_token(q, k, v, w_q.contiguous(), w_k.contiguous(), table, **kw)
    else:
        out = engine.forward(q, k, v, w_q.contiguous(), w_k.contiguous(), table, local=not sequence, **kw)
    if sequence and state.get("ulysses", True):
        state["ulysses_local_heads"] = -(-heads // engine.world_rank()[0])
    return self.out_proj(out.reshape(n, heads * dim).to(x.dtype if x.is_floating_point() else out.dtype))


def install_attention(module, group=None, state: dict | None = None):
    """Route one H3 Attention module through the b200 path (the counterpart of
    powershard/attention.py:184-195 for a single module)."""
    module.forward = types.MethodType(attention_forward, module)
    module._ps_b200_group = group
    if state is not None:
        module._ps_sequence = state
    return module
