"""CPU oracle for the Ulysses sequence-parallel attention path (TEST INFRASTRUCTURE).

This module restates, in plain PyTorch on the CPU, the algorithm PowerShard
(ComfyUI-PowerShard v0.6.0) runs for one Wan self-attention block in
``sequence_mode="ulysses"``.  It is the checker for the CUDA product path and
the timed CPU baseline of ``bench.py``; nothing in the product imports it.
Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its
``cpu_baseline`` leg and ``--impl reference`` arm) may use it.

Parity pinning: ``tests/golden/make_golden.py`` imported the reference
package from its source tree and recorded its outputs (RMSNorm, rope_apply,
attention_qkv, ulysses_to_sequence / ulysses_to_heads over emulated
collectives, math_attention, sequence_attention in Ulysses and token mode,
image_parallel's
SequenceAttention over an image_layout.Layout) as fixtures under
``tests/golden/``; ``tests/test_oracle_golden.py`` checks every function here
against them.  One piece is NOT pinned: the 3-D RoPE *table*
(``rope_table_3d``) restates ComfyUI's ``WanModel.rope_encode`` (ComfyUI sha
7a0b5eede3f9721c8faab290689893f36edc6d66), which is not part of the
reference tree; only its consumer ``rope_apply`` and the axis split are.

Reference line citations are paths inside the ComfyUI-PowerShard project.
"""
from __future__ import annotations

import math
import time

import torch
import torch.nn.functional as F

__all__ = [
    "shard_bounds", "rms_norm", "rope_apply", "rope_split_half", "rope_axes", "rope_table_3d",
    "rope_table_flux", "attention_qkv", "pack_qkv", "exchange", "unpack_qkv",
    "pack_out", "unpack_out", "math_attention", "sdpa_fp32", "sequence_attention", "gather_rows",
    "token_sequence_attention",
    "rms_norm_heads", "flux_joint_attention", "split_sizes", "image_local_ranges",
    "image_sequence_attention", "time_reference_sample", "time_reference_step",
]


# ----------------------------------------------------------------- partition
def shard_bounds(rows: int, rank: int, world_size: int):
    """Ceil-width contiguous token shard [a, b); last ranks may be empty.

    Follows powershard/config.py:107-112 (Shard(0) / torch.chunk semantics).
    """
    if rows < 0 or world_size < 1 or not 0 <= rank < world_size:
        raise ValueError("invalid shard bounds")
    width = (rows + world_size - 1) // world_size
    return min(rows, rank * width), min(rows, (rank + 1) * width)


# ------------------------------------------------------------ norm and RoPE
def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """fp32 RMSNorm over the last axis, cast back to x.dtype.

    Follows powershard/operations.py:61-64 (``RMSNorm.forward``): the
    statistic is the mean of squares of the fp32 values, the weight is
    applied in fp32, the result is rounded once to the input dtype.
    """
    y = x.float()
    y = y * torch.rsqrt(y.square().mean(-1, keepdim=True) + eps)
    return (y * weight.float()).to(x.dtype)


def rope_apply(x: torch.Tensor, freqs: torch.Tensor) -> torch.Tensor:
    """[B,L,H,D] x [1,L,1,D/2,2,2] -> fp32 [B,L,H,D], interleaved pairs.

    Follows powershard/wan_model.py:325-329: for pair j = (x[2j], x[2j+1])
    out[2j]   = F[j,0,0]*x[2j] + F[j,0,1]*x[2j+1]
    out[2j+1] = F[j,1,0]*x[2j] + F[j,1,1]*x[2j+1]
    with each product rounded in fp32 before the sum.
    """
    # Explicit pair count instead of the reference's -1 so empty shards work.
    x_ = x.float().reshape(*x.shape[:-1], x.shape[-1] // 2, 1, 2)
    out = freqs[..., 0] * x_[..., 0] + freqs[..., 1] * x_[..., 1]
    return out.reshape(*x.shape)


def rope_split_half(x: torch.Tensor, table: torch.Tensor) -> torch.Tensor:
    """H3 partial RoPE: [S,H,D] x [1,S,1,P,2,2] (powershard/attention.py:98-103).

    Element j < P pairs with element j+P: out_j = M00 x_j + M01 x_{j+P},
    out_{j+P} = M10 x_j + M11 x_{j+P} (fp32), elements >= 2P pass through;
    the result is cast back to x.dtype.
    """
    p = table.shape[-3]
    m = table[0].float()
    a, b = x[..., :p].float(), x[..., p:2 * p].float()
    first = m[..., 0, 0] * a + m[..., 0, 1] * b
    second = m[..., 1, 0] * a + m[..., 1, 1] * b
    return torch.cat([first, second, x[..., 2 * p:].float()], -1).to(x.dtype)


def rope_axes(head_dim: int):
    """(t, h, w) RoPE dims: head_dim - 4*(head_dim//6), 2*(head_dim//6) twice.

    Follows powershard/wan_model.py:1199 (44/42/42 for head_dim 128).
    """
    third = head_dim // 6
    return head_dim - 4 * third, 2 * third, 2 * third


def _rope_axis(pos: torch.Tensor, dim: int, theta: float) -> torch.Tensor:
    # Standard RoPE: omega_k = theta^(-2k/dim), k in [0, dim/2); 2x2 rotation
    # [[cos, -sin], [sin, cos]] per pair (published Flux/Wan EmbedND form).
    scale = torch.arange(0, dim, 2, dtype=torch.float64) / dim
    omega = 1.0 / (theta ** scale)
    ang = pos.to(torch.float64)[:, None] * omega[None, :]
    c, s = torch.cos(ang), torch.sin(ang)
    return torch.stack([c, -s, s, c], dim=-1).reshape(pos.shape[0], dim // 2, 2, 2).float()


def rope_table_3d(grid, head_dim: int = 128, theta: float = 10000.0) -> torch.Tensor:
    """[1, T*H*W, 1, head_dim/2, 2, 2] fp32 table for a (t, h, w) token grid.

    Tokens are ordered row-major over (t, h, w).  Pairs [0, dt/2) rotate by
    the t index, the next dh/2 by h, the last dw/2 by w (axes from
    ``rope_axes``).  Restates ComfyUI ``WanModel.rope_encode`` (not in the
    reference tree): parity of this table is unpinned.
    """
    T, Hg, Wg = grid
    dt, dh, dw = rope_axes(head_dim)
    t = torch.arange(T).repeat_interleave(Hg * Wg)
    h = torch.arange(Hg).repeat_interleave(Wg).repeat(T)
    w = torch.arange(Wg).repeat(T * Hg)
    table = torch.cat([_rope_axis(t, dt, theta), _rope_axis(h, dh, theta),
                       _rope_axis(w, dw, theta)], dim=1)
    return table[None, :, None]


def rope_table_flux(text_tokens: int, grid_hw, head_dim: int = 128,
                    axes=(16, 56, 56), theta: float = 10000.0) -> torch.Tensor:
    """Flux joint table: text ids are 0 (identity), image ids (0, h, w).

    Restates the ComfyUI Flux EmbedND (not in the reference tree): unpinned.
    """
    Hg, Wg = grid_hw
    n_img = Hg * Wg
    ids = torch.zeros(text_tokens + n_img, 3, dtype=torch.int64)
    ids[text_tokens:, 1] = torch.arange(Hg).repeat_interleave(Wg)
    ids[text_tokens:, 2] = torch.arange(Wg).repeat(Hg)
    parts = [_rope_axis(ids[:, i], d, theta) for i, d in enumerate(axes)]
    return torch.cat(parts, dim=1)[None, :, None]


def attention_qkv(q_lin, k_lin, v_lin, wq, wk, freqs, heads: int, eps: float = 1e-6):
    """Wan q/k/v from projection outputs [B,n,H*D]: fp32 q, k and v [B,n,H,D].

    Follows powershard/wan_model.py:421-430: q = rope_apply(norm_q(q).view),
    k likewise, v = v.view (no norm, no rotation).
    """
    b, n, width = q_lin.shape
    dim = width // heads
    k = rope_apply(rms_norm(k_lin, wk, eps).view(b, n, heads, dim), freqs)
    v = v_lin.view(b, n, heads, dim)
    q = rope_apply(rms_norm(q_lin, wq, eps).view(b, n, heads, dim), freqs)
    return q, k, v


# ---------------------------------------------------------- Ulysses exchange
def pack_qkv(q, k, v, total: int, rank: int, world: int):
    """Send buffer [W(dst), 3, width, h, D] of one rank (batch 1, LHD rows).

    Follows powershard/attention.py:57-75 and wan_model.py:343-361: heads are
    zero-padded to h*W (h = ceil(H/W)), tokens to width = ceil(total/W);
    destination r receives heads [r*h, (r+1)*h) of all local tokens.
    """
    width, h = math.ceil(total / world), math.ceil(q.shape[1] / world)
    a, b = shard_bounds(total, rank, world)
    n, heads, dim = q.shape
    if n != b - a:
        raise ValueError("local token count does not match shard_bounds")
    parts = []
    for t in (q, k, v):
        padded = t.new_zeros((width, h * world, dim))
        padded[:n, :heads] = t
        parts.append(padded.view(width, world, h, dim).transpose(0, 1))
    return torch.stack(parts, dim=1).contiguous()


def exchange(sends):
    """all_to_all_single over dim 0: recv[r][s] = send[s][r] for every rank."""
    world = len(sends)
    return [torch.stack([sends[s][r] for s in range(world)]) for r in range(world)]


def unpack_qkv(recv, total: int):
    """[W(src), 3, width, h, D] -> (q, k, v) each [total, h, D].

    Follows powershard/attention.py:77-79: sources are concatenated in rank
    order and token padding (only at the tail) is removed with [:total].
    """
    world, three, width, h, dim = recv.shape
    full = recv.permute(1, 0, 2, 3, 4).reshape(three, world * width, h, dim)
    return tuple(t[:total] for t in full)


def pack_out(out, total: int, world: int):
    """[total, h, D] -> send [W(dst), width, h, D] (powershard/attention.py:82-93)."""
    width = math.ceil(total / world)
    padded = out.new_zeros((world * width,) + tuple(out.shape[1:]))
    padded[:total] = out
    return padded.view(world, width, *out.shape[1:])


def unpack_out(recv, total: int, heads: int, rank: int, world: int):
    """[W(src), width, h, D] -> [n_local, H, D], dropping padded heads.

    Follows powershard/attention.py:93-95 / wan_model.py:379-380.
    """
    a, b = shard_bounds(total, rank, world)
    _, width, h, dim = recv.shape
    return recv.transpose(0, 1)[:b - a].reshape(b - a, world * h, dim)[:, :heads].contiguous()


# --------------------------------------------------------------- attention
def math_attention(q, k, v, scale=None, query_chunk: int = 128, key_chunk: int = 512):
    """Tiled fp32 online-softmax attention, BLHD in and out (non-causal, no mask).

    Follows powershard/attention_contract.py:85-125 for the options the
    Ulysses path uses (no mask/causal/window/ALiBi/dropout): per query chunk
    a running max m, denominator den and accumulator acc over key chunks;
    fully masked rows (den == 0) are divided by 1.  Output dtype = q.dtype.
    """
    b, lq, h, d = q.shape
    qh, kh, vh = (x.transpose(1, 2) for x in (q, k, v))
    scale = d ** -0.5 if scale is None else scale
    output = torch.empty((b, h, lq, v.shape[-1]), dtype=q.dtype)
    for a in range(0, lq, query_chunk):
        z = min(a + query_chunk, lq)
        qs = qh[..., a:z, :].float()
        m = torch.full((b, h, z - a, 1), -torch.inf)
        den = torch.zeros_like(m)
        acc = torch.zeros((b, h, z - a, v.shape[-1]))
        for c in range(0, kh.shape[-2], key_chunk):
            e = min(c + key_chunk, kh.shape[-2])
            scores = (qs @ kh[..., c:e, :].float().transpose(-1, -2)) * scale
            new_m = torch.maximum(m, scores.amax(-1, keepdim=True))
            safe_m = torch.where(new_m == -torch.inf, 0.0, new_m)
            alpha = torch.exp(m - safe_m)
            p = torch.exp(scores - safe_m)
            acc = acc * alpha + p @ vh[..., c:e, :].float()
            den = den * alpha + p.sum(-1, keepdim=True)
            m = new_m
        output[..., a:z, :] = acc / torch.where(den == 0, 1.0, den)
    return output.transpose(1, 2).contiguous()


def sdpa_fp32(q, k, v, scale=None):
    """Reference provider of the north star: fp32 SDPA math path, BLHD.

    powershard/attention_contract.py:128-145 with fp32 inputs; evaluated
    here as an explicit softmax(QK^T*scale)V in fp32 (the SDPA math kernel).
    """
    qf, kf, vf = (x.float().transpose(1, 2) for x in (q, k, v))
    scale = q.shape[-1] ** -0.5 if scale is None else scale
    out = F.scaled_dot_product_attention(qf, kf, vf, scale=scale)
    return out.transpose(1, 2).contiguous()


# ------------------------------------------------------------- whole path
def _power2_scale(ratio: torch.Tensor) -> torch.Tensor:
    """2^ceil(log2(max(ratio, 1))) (powershard/fp16_safe.py:18-20)."""
    return torch.exp2(torch.ceil(torch.log2(torch.maximum(ratio, torch.ones_like(ratio)))))


def sequence_attention(q_lin, k_lin, v_lin, wq, wk, freqs, heads: int, world: int,
                       eps: float = 1e-6, wire_dtype=torch.bfloat16, attention="sdpa",
                       scale=None, provider_dtype=None, v_scales=None):
    """Whole Ulysses self-attention of one block, all ranks simulated in-process.

    Inputs are the GLOBAL projection outputs [1, L, H*D] and the global RoPE
    table [1, L, 1, D/2, 2, 2]; rank r owns tokens shard_bounds(L, r, W).
    Per rank (powershard/wan_model.py:421-430, 441-502):
      attention_qkv -> cast to the wire dtype -> pack [W,3,width,h,D]
      -> all_to_all -> attention over all L tokens for h heads
      -> pack [W,width,h,D] -> all_to_all -> [n, H, D].
    Returns the list of per-rank outputs [1, n_r, H, D] in the wire dtype
    (attention computed in fp32, rounded once to the wire dtype).

    provider_dtype reproduces run_attention (wan_model.py:398-418): q/k are
    cast to that dtype, v divided by its power-of-two scale sv before the
    cast, the provider output rounded to it and multiplied back by sv.  The
    reference takes sv over everything one call receives (v_scale,
    wan_model.py:389-395), so a batch of rows shares it: ``v_scales`` (one
    scalar tensor per rank) supplies that shared scale when this function
    is called one batch row at a time.
    """
    total = q_lin.shape[1]
    sends = []
    for r in range(world):
        a, b = shard_bounds(total, r, world)
        q, k, v = attention_qkv(q_lin[:, a:b], k_lin[:, a:b], v_lin[:, a:b], wq, wk,
                                freqs[:, a:b], heads, eps)
        sends.append(pack_qkv(q[0].to(wire_dtype), k[0].to(wire_dtype),
                              v[0].to(wire_dtype), total, r, world))
    recvs = exchange(sends)
    outs = []
    for r in range(world):
        q, k, v = unpack_qkv(recvs[r], total)
        fn = sdpa_fp32 if attention == "sdpa" else math_attention
        if provider_dtype is None:
            o = fn(q[None].float(), k[None].float(), v[None].float(), scale)[0]
        else:
            if v_scales is not None:
                sv = v_scales[r]
            else:
                sv = _power2_scale(v.float().abs().amax() / 16384.0) if v.numel() else torch.ones(())
            o = fn(q[None].float().to(provider_dtype), k[None].float().to(provider_dtype),
                   (v[None].float() / sv).to(provider_dtype), scale)[0]
            o = o.to(provider_dtype).float() * sv
        outs.append(pack_out(o.to(wire_dtype), total, world))
    back = exchange(outs)
    return [unpack_out(back[r], total, heads, r, world)[None] for r in range(world)]


def gather_rows(parts, total: int, world: int):
    """All-gather of token rows (powershard/attention.py:40-54): each rank's
    rows padded to ceil(total/W), concatenated in rank order, sliced to total."""
    width = math.ceil(total / world)
    padded = []
    for p in parts:
        z = p.new_zeros((width,) + tuple(p.shape[1:]))
        z[:p.shape[0]] = p
        padded.append(z)
    return torch.cat(padded)[:total]


def token_sequence_attention(q_lin, k_lin, v_lin, wq, wk, freqs, heads: int, world: int, eps: float = 1e-6,
                             attention="sdpa", scale=None, provider_dtype=None):
    """Token-mode self-attention of one block (sequence_mode="token"), ranks
    simulated: per rank attention_qkv of its rows (powershard/wan_model.py:
    421-430), k/v of every rank gathered (gather_tokens, :336-340, over
    gather_rows), run_attention (:398-418) of the local queries against all
    keys (:489-500).  Returns per rank the fp32 output [1, n_r, H, D];
    provider_dtype as in ``sequence_attention``."""
    total = q_lin.shape[1]
    local = []
    for r in range(world):
        a, b = shard_bounds(total, r, world)
        local.append(attention_qkv(q_lin[:, a:b], k_lin[:, a:b], v_lin[:, a:b], wq, wk, freqs[:, a:b], heads, eps))
    k = gather_rows([t[1][0] for t in local], total, world)[None]
    v = gather_rows([t[2][0] for t in local], total, world)[None]
    fn = sdpa_fp32 if attention == "sdpa" else math_attention
    outs = []
    for r in range(world):
        q = local[r][0]
        if q.shape[1] == 0:
            outs.append(q.new_zeros(q.shape, dtype=torch.float32))
            continue
        if provider_dtype is None:
            outs.append(fn(q.float(), k.float(), v.float(), scale))
        else:
            sv = _power2_scale(v.float().abs().amax() / 16384.0)
            o = fn(q.float().to(provider_dtype), k.float().to(provider_dtype),
                   (v.float() / sv).to(provider_dtype), scale)
            outs.append(o.to(provider_dtype).float() * sv)
    return outs


# ------------------------------------------------- Flux joint attention
def rms_norm_heads(x, weight, heads: int, eps: float = 1e-6):
    """Per-head RMSNorm (Flux QK-norm): [B,n,H*D] -> [B,n,H,D], weight [D].

    Same fp32-statistic / cast-back semantics as operations.RMSNorm
    (powershard/operations.py:61-64), applied over each head's D values.
    Restates ComfyUI's Flux QKNorm (not in the reference tree): unpinned.
    """
    b, n, width = x.shape
    y = x.view(b, n, heads, width // heads).float()
    y = y * torch.rsqrt(y.square().mean(-1, keepdim=True) + eps)
    return (y * weight.float()).to(x.dtype)


def flux_joint_attention(txt, img, wq, wk, txt_freqs, img_freqs, heads: int, world: int, eps: float = 1e-6,
                         wire_dtype=torch.bfloat16, scale=None):
    """Flux joint attention of one double/single block, ranks simulated.

    txt = (q, k, v) [1, P, H*D] text projections (replicated on every rank),
    img = (q, k, v) [1, L, H*D] image projections (rank r owns
    shard_bounds(L, r, W)); freqs tables [1, n, 1, D/2, 2, 2].  Keys and
    queries are [text; image] (powershard/image_parallel.py:96-110 computes
    the same attention with a K/V all-gather).  Returns per rank
    (text out [P, H, D], image out [n_r, H, D]) in the wire dtype.
    """
    def qk(x, w, f):
        return rope_apply(rms_norm_heads(x, w, heads, eps), f).to(wire_dtype)
    q = torch.cat([qk(txt[0], wq, txt_freqs), qk(img[0], wq, img_freqs)], 1)
    k = torch.cat([qk(txt[1], wk, txt_freqs), qk(img[1], wk, img_freqs)], 1)
    p, d = txt[2].shape[1], txt[2].shape[2] // heads
    v = torch.cat([txt[2].view(1, p, heads, d), img[2].view(1, -1, heads, d)], 1).to(wire_dtype)
    out = sdpa_fp32(q, k, v, scale)[0].to(wire_dtype)
    total = img[0].shape[1]
    res = []
    for r in range(world):
        a, b = shard_bounds(total, r, world)
        res.append((out[:p], out[p + a:p + b]))
    return res


# ------------------------------------- image Layout sequence attention
def split_sizes(n: int, world: int):
    """Balanced split of n rows: the first n % world ranks get one extra row
    (powershard/image_layout.py:12-15)."""
    base, extra = divmod(int(n), int(world))
    return [base + (1 if r < extra else 0) for r in range(int(world))]


def image_local_ranges(segments, world: int, rank: int):
    """Global row ranges that make up `rank`'s local sequence for segments
    [(rows, split)] with exactly one split segment: all rows before the split
    segment, the rank's part [a, b) of its balanced split, all rows after it
    (powershard/image_layout.py:22-49)."""
    total = sum(int(n) for n, _ in segments)
    start = 0
    for n, split in segments:
        if split:
            split_start, split_len = start, int(n)
        start += int(n)
    sizes = split_sizes(split_len, world)
    a = split_start + sum(sizes[:rank])
    b = a + sizes[rank]
    out = []
    if split_start > 0:
        out.append((0, split_start))
    if b > a:
        out.append((a, b))
    if split_start + split_len < total:
        out.append((split_start + split_len, total))
    return out


def image_sequence_attention(q, k, v, segments, world: int, scale=None):
    """What powershard/image_parallel.py:96-110 (SequenceAttention.__call__)
    returns on every rank: the rank's local query rows (image_local_ranges)
    attend over the full key/value sequence that assemble_full (:45-52)
    rebuilds by all-gathering the split segment.  q, k, v: full [B, L, H, D];
    returns per rank the fp32 output [B, n_local, H, D] of those rows."""
    out = sdpa_fp32(q, k, v, scale)
    res = []
    for r in range(world):
        rows = [i for s, e in image_local_ranges(segments, world, r) for i in range(s, e)]
        res.append(out[:, rows])
    return res


# ------------------------------------------------------ timed CPU baseline
def time_reference_sample(total: int, heads: int, dim: int, budget_s: float = 12.0,
                          threads: int | None = None, seed: int = 0):
    """Time the reference's CPU algorithm on a bounded sample of one layer.

    The sample is: the full per-token pre-pass (RMSNorm + RoPE + pack) for
    all ``total`` tokens, then ``math_attention`` (128x512 fp32 tiles, the
    reference default provider) over query chunks of head 0 against all
    ``total`` keys until ``budget_s`` seconds are spent.  The attention time
    is extrapolated linearly to all query chunks of all heads.

    Returns a dict with the extrapolated seconds per layer, TFLOP/s over the
    layer's 4*L^2*H*D attention FLOPs, the measured sample and threads used.
    """
    if threads:
        torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(seed)
    width = heads * dim
    # Pre-pass over every token, in chunks to bound host memory.
    t0 = time.perf_counter()
    chunk = 4096
    w = torch.ones(width)
    grid_tokens = total
    freqs_cache = None
    for a in range(0, total, chunk):
        z = min(a + chunk, total)
        xs = [torch.randn(1, z - a, width, generator=g) for _ in range(3)]
        if freqs_cache is None or freqs_cache.shape[1] != z - a:
            ang = torch.randn(1, z - a, 1, dim // 2, generator=g)
            c, s = torch.cos(ang), torch.sin(ang)
            freqs_cache = torch.stack([c, -s, s, c], -1).reshape(1, z - a, 1, dim // 2, 2, 2)
        q, k, v = attention_qkv(xs[0], xs[1], xs[2], w, w, freqs_cache, heads)
        pack_qkv(q[0], k[0], v[0], z - a, 0, 1)
    prepass_s = time.perf_counter() - t0
    # Attention sample: head 0, query chunks of 128 against all keys.
    kk = torch.randn(1, grid_tokens, 1, dim, generator=g)
    vv = torch.randn(1, grid_tokens, 1, dim, generator=g)
    done_chunks = 0
    t1 = time.perf_counter()
    while True:
        qq = torch.randn(1, 128, 1, dim, generator=g)
        math_attention(qq, kk, vv)
        done_chunks += 1
        if time.perf_counter() - t1 > budget_s or done_chunks * 128 >= grid_tokens * heads:
            break
    attn_sample_s = time.perf_counter() - t1
    all_chunks = math.ceil(grid_tokens / 128) * heads
    attn_s = attn_sample_s / done_chunks * all_chunks
    layer_s = prepass_s + attn_s
    flops = 4.0 * total * total * heads * dim
    return dict(seconds_per_layer=layer_s, tflops=flops / layer_s / 1e12,
                prepass_s=prepass_s, attention_sample_s=attn_sample_s,
                attention_chunks=done_chunks, attention_chunks_total=all_chunks,
                threads=torch.get_num_threads())


def time_reference_step(total: int, heads: int, dim: int, budget_s: float = 5.0,
                        threads: int | None = None, seed: int = 0):
    """One measured step of the reference's CPU algorithm on a bounded,
    proportional slice of one layer (nothing extrapolated inside the step).

    The step runs ``math_attention`` (128x512 fp32 tiles, the reference's
    default provider, powershard/attention_contract.py:85-125) for query
    chunks of 128 rows of one head against all ``total`` keys until
    ``budget_s`` is spent - c chunks, the fraction f = c / (ceil(L/128)*H) of
    the layer's attention - and then the per-token pre-pass (attention_qkv +
    pack, powershard/wan_model.py:421-430 and 343-361) over the same fraction
    f of the tokens.  Both parts scale linearly with f, so the step's rate
    (attention FLOPs executed / wall time of the step) is the layer's rate.

    Returns the step's wall seconds, the FLOPs it executed (4*128*c*L*D),
    their rate, the chunks and tokens processed and the threads used.
    """
    if threads:
        torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(seed)
    width = heads * dim
    all_chunks = math.ceil(total / 128) * heads
    kk = torch.randn(1, total, 1, dim, generator=g)
    vv = torch.randn(1, total, 1, dim, generator=g)
    queries = [torch.randn(1, 128, 1, dim, generator=g) for _ in range(4)]
    t0 = time.perf_counter()
    chunks = 0
    while True:
        math_attention(queries[chunks % 4], kk, vv)
        chunks += 1
        if time.perf_counter() - t0 > budget_s or chunks >= all_chunks:
            break
    attn_s = time.perf_counter() - t0
    tokens = max(1, round(total * chunks / all_chunks))
    xs = [torch.randn(1, tokens, width, generator=g) for _ in range(3)]
    ang = torch.rand(1, tokens, 1, dim // 2, generator=g) * 40.0
    c, s = torch.cos(ang), torch.sin(ang)
    freqs = torch.stack([c, -s, s, c], -1).reshape(1, tokens, 1, dim // 2, 2, 2)
    w = torch.ones(width)
    t1 = time.perf_counter()
    q, k, v = attention_qkv(xs[0], xs[1], xs[2], w, w, freqs, heads)
    pack_qkv(q[0], k[0], v[0], tokens, 0, 1)
    prepass_s = time.perf_counter() - t1
    wall = attn_s + prepass_s
    flops = 4.0 * 128 * chunks * total * dim
    return dict(wall_s=wall, flops=flops, tflops=flops / wall / 1e12, attention_s=attn_s,
                prepass_s=prepass_s, chunks=chunks, chunks_total=all_chunks, tokens=tokens,
                fraction=chunks / all_chunks, threads=torch.get_num_threads())
