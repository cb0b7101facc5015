"""Wan self-attention entry points with the PowerShard signatures.

* ``self_attention_forward(self, x, freqs, transformer_options=None)`` -
  replacement for powershard/wan_model.py:433-438.  When q/k/v/o are plain
  Linear layers (the reference's Linear without its scaled-fp16 path) the
  whole layer runs in the fused kernels (``UlyssesAttention.forward_layer``:
  q/k/v GEMM with RMSNorm + RoPE + pack in its epilogue, attention, output
  GEMM reading the exchange buffer); otherwise the projections stay the
  module's own layers and q/k RMSNorm + RoPE run fused with the pack.
* ``sequence_attention(self, q, k, v, total=None)`` - replacement for
  powershard/wan_model.py:441-502 for callers that already produced
  normalised, rotated q/k (the pre-pass then only packs).

Both follow the shared state's mode: Ulysses (``ulysses`` true, the
default) or token mode (K/V all-gathered, local queries,
wan_model.py:489-500).  ``gather_tokens`` is the final-head gather of the
sequence-parallel forward (wan_model.py:336-340, :1072-1075).

Both read the module attributes the reference installs
(``install_wan_compute``, wan_model.py:727-768): ``num_heads``,
``head_dim``, ``_ps_sequence`` (the shared state dict: ``enabled``,
``ulysses``, ``total`` ...), and update the same counters
(``kv_collectives``, ``kv_gathered_bytes``, ``out_collectives``,
``out_exchanged_bytes``, ``padded_heads``, ``effective_comm_dtype``).
The sequence-parallel process group is ``_ps_b200_group`` (None = default).
"""
from __future__ import annotations

import types

import torch
import torch.distributed as dist

from . import ops
from .contract import AttentionOptions, UnsupportedAttention
from .partition import shard_bounds
from .ulysses import UlyssesAttention

WIRE_DTYPE = torch.bfloat16


def _engine(module) -> UlyssesAttention:
    engine = getattr(module, "_ps_b200_engine", None)
    if engine is None:
        engine = UlyssesAttention(getattr(module, "_ps_b200_group", None))
        module._ps_b200_engine = engine
    return engine


def _state(module) -> dict:
    state = getattr(module, "_ps_sequence", None)
    if state is None:
        state = dict(total=0, enabled=False, ulysses=True, comm_dtype="bf16", mode="ulysses")
        module._ps_sequence = state
    return state


def _check_supported(module, state):
    if getattr(module, "_ps_main", False) and state.get("ref_attn_masks") is not None:
        raise UnsupportedAttention("b200: InfiniteTalk reference attention maps are not provided")


def _rows(t, heads, head_dim, dtype):
    """[B, n, H, D] or [B, n, H*D] -> [B, n, H*D] in the wire dtype with unit
    inner stride and 16-byte aligned rows (a copy only when needed)."""
    t = t.reshape(t.shape[0], t.shape[1], heads * head_dim)
    if t.dtype != dtype:
        t = t.to(dtype)
    if t.stride(-1) != 1 or any(st % 8 for st in t.stride()[:-1]) or t.data_ptr() % 16:
        t = t.contiguous()
    return t


def _run(engine, state, q, k, v, w_q, w_k, table, total, heads, norm_rope, out_dtype, local, eps=1e-6):
    """The batch [B, n, H*D] through Ulysses (one exchange for the whole batch)
    or token mode (the shared state's ``ulysses`` flag); counters once per call."""
    token = state.get("enabled") and not state.get("ulysses", True)
    counted = state if state.get("enabled") else None
    if not token:
        return engine.forward_batch(q, k, v, w_q, w_k, table, total=total, heads=heads, eps=eps,
                                    norm_rope=norm_rope, out_dtype=out_dtype, state=counted, local=local)
    outs = [engine.forward_token(q[b], k[b], v[b], w_q, w_k,
                                 table[b] if table is not None and table.dim() == 5 else table,
                                 total=total, heads=heads, eps=eps, norm_rope=norm_rope, out_dtype=out_dtype)
            for b in range(q.shape[0])]
    if counted is not None:
        # The reference gathers the whole batch's K/V in one all-gather
        # (wan_model.py:489-493): one collective, the batch's bytes.
        engine.count_token(counted, total, heads, q.shape[-1] // heads, q.dtype, engine.last_exchange,
                           batch=q.shape[0])
    return torch.stack(outs)


def _plain_linear(lin) -> bool:
    """A Linear layer whose forward is x W^T + b: torch's, or the reference's
    operations.Linear outside its scaled-fp16 / prepared-int8 paths."""
    return (isinstance(lin, torch.nn.Linear) and not getattr(lin, "_ps_safe", False)
            and getattr(lin, "_ps_prepared", None) is None and lin.weight.dim() == 2)


def _fused_layers(module, dtype):
    """(w_q, w_k, w_v, w_o, b_q, b_k, b_v, b_o) for the fused layer, or None
    when the layer shape or the Linear layers do not fit it.  The weights
    must already be in the wire dtype: a 16-bit Linear casts its input to its
    weight dtype, as the fused GEMM does, while layers kept in fp32 keep their
    own fp32 projections (the fused path never lowers their precision)."""
    if not getattr(module, "_ps_b200_fused_projections", True):
        return None
    lins = [getattr(module, name, None) for name in "qkvo"]
    if not all(_plain_linear(lin) and lin.weight.is_cuda and lin.weight.dtype == dtype for lin in lins):
        return None
    heads, dim = module.num_heads, module.head_dim
    width = heads * dim
    fin = lins[0].weight.shape[1]
    if (dim != 128 or width % 256 or fin % 64 or lins[3].weight.shape[0] % 256 or lins[3].weight.shape[1] != width
            or any(tuple(lin.weight.shape) != (width, fin) for lin in lins[:3])):
        return None
    key = tuple((lin.weight.data_ptr(), lin.weight._version,
                 None if lin.bias is None else (lin.bias.data_ptr(), lin.bias._version)) for lin in lins) + (dtype,)
    cached = getattr(module, "_ps_b200_fused_cache", None)
    if cached is not None and cached[0] == key:
        return cached[1]
    weights = [lin.weight.detach().contiguous() for lin in lins]
    biases = [None if lin.bias is None else lin.bias.detach().float().contiguous() for lin in lins]
    value = (*weights, *biases)
    module._ps_b200_fused_cache = (key, value)
    return value


def self_attention_forward(self, x, freqs, transformer_options=None):
    """x [B, n, dim] -> [B, n, dim] through the fused Ulysses path (the whole
    batch in one exchange, as the reference)."""
    state = _state(self)
    _check_supported(self, state)
    batch, n, _ = x.shape
    heads, dim = self.num_heads, self.head_dim
    total = state["total"] if state.get("enabled") else n
    engine = _engine(self)
    # The reference's table [1 or B, n, 1, D/2, 2, 2] (wan_model.py:325-329):
    # one table shared by the batch rows, or one per row.
    table = freqs[:, :, 0] if freqs.shape[0] > 1 else freqs[0, :, 0]
    if table.dtype != torch.float32 or table.stride()[-3:] != (4, 2, 1) or table.data_ptr() % 16:
        table = table.float().contiguous()
    w_q = self.norm_q.weight
    w_k = self.norm_k.weight
    if w_q.dtype not in (torch.float32, WIRE_DTYPE):
        w_q, w_k = w_q.float(), w_k.float()
    eps = self.norm_q.eps if self.norm_q.eps is not None else 1e-6
    token = state.get("enabled") and not state.get("ulysses", True)
    fused = None if token or not x.is_cuda or engine.kernels is not ops else _fused_layers(self, WIRE_DTYPE)
    if fused is not None:
        # The whole layer in the fused kernels: no projection or attention
        # output makes a separate round trip through memory.
        out_dtype = x.dtype if x.is_floating_point() else WIRE_DTYPE
        return engine.forward_layer(x.to(WIRE_DTYPE), *fused[:4], w_q.contiguous(), w_k.contiguous(), table,
                                    *fused[4:], total=total, heads=heads, eps=eps, out_dtype=out_dtype,
                                    state=state if state.get("enabled") else None, local=not state.get("enabled"))
    q_lin, k_lin, v_lin = self.q(x), self.k(x), self.v(x)
    out = _run(engine, state, _rows(q_lin, heads, dim, WIRE_DTYPE), _rows(k_lin, heads, dim, WIRE_DTYPE),
               _rows(v_lin, heads, dim, WIRE_DTYPE), w_q.contiguous(), w_k.contiguous(), table, total, heads,
               True, None, not state.get("enabled"), eps)
    return self.o(out.reshape(batch, n, heads * dim).to(x.dtype if x.is_floating_point() else out.dtype))


def sequence_attention(self, q, k, v, total=None):
    """q, k, v [B, n, H, D] (already RMSNorm'd and rotated) -> [B, n, H, D] fp32."""
    state = _state(self)
    _check_supported(self, state)
    batch, n, heads, dim = q.shape
    if not state.get("enabled"):
        from .provider import B200Provider
        provider = getattr(self, "_ps_b200_provider", None) or B200Provider()
        self._ps_b200_provider = provider
        out = provider(q.to(WIRE_DTYPE), k.to(WIRE_DTYPE), v.to(WIRE_DTYPE),
                       AttentionOptions(softmax_scale=dim ** -0.5))
        return out.float()
    total = total or state["total"]
    engine = _engine(self)
    return _run(engine, state, _rows(q, heads, dim, WIRE_DTYPE), _rows(k, heads, dim, WIRE_DTYPE),
                _rows(v, heads, dim, WIRE_DTYPE), None, None, None, total, heads, False, torch.float32, False)


def gather_tokens(x, total, dtype=None, group=None):
    """Batch-first all-gather of token rows: [B, n, ...] -> [B, total, ...].

    The final-head gather of the sequence-parallel Wan forward
    (powershard/wan_model.py:336-340, called at :1072-1075, where the caller
    counts ``head_gathers``), with the row semantics of
    powershard/attention.py:40-54: rank r holds rows shard_bounds(total, r,
    W); every rank's rows are padded to ceil(total / W), one
    all_gather_into_tensor (NCCL on the current stream for CUDA tensors)
    concatenates them in rank order, and the padding is cut.  `dtype` is the
    wire dtype; the result comes back in x's dtype.  The result is a fresh
    tensor, never a view of a buffer that a later call rewrites.
    """
    world, rank = (dist.get_world_size(group), dist.get_rank(group)) if dist.is_initialized() else (1, 0)
    a, b = shard_bounds(total, rank, world)
    if x.shape[1] != b - a:
        raise ValueError(f"gather_tokens: {x.shape[1]} local tokens, shard_bounds gives {b - a}")
    wire = dtype or x.dtype
    width = -(-total // world)
    rows = x.transpose(0, 1)                       # [n, B, ...] view
    send = torch.zeros((width,) + tuple(rows.shape[1:]), dtype=wire, device=x.device)
    send[:b - a].copy_(rows)
    gathered = torch.empty((world * width,) + tuple(rows.shape[1:]), dtype=wire, device=x.device)
    if world > 1:
        dist.all_gather_into_tensor(gathered, send, group=group)
    else:
        gathered.copy_(send)
    return gathered[:total].transpose(0, 1).to(x.dtype).contiguous()


def install_self_attention(module, group=None, state: dict | None = None):
    """Route one WanSelfAttention-like module through the b200 path.

    The counterpart of the ``"self"`` branch of install_wan_compute
    (powershard/wan_model.py:740-746): replaces ``module.forward`` and
    attaches the shared sequence state and process group.
    """
    module.forward = types.MethodType(self_attention_forward, module)
    module._ps_b200_group = group
    if state is not None:
        module._ps_sequence = state
    return module
