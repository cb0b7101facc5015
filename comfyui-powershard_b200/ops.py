"""Tensor-level wrappers of the three device steps (one C-ABI call each).

Each wrapper checks devices, dtypes, shapes and contiguity, then calls the
matching ``ps_b200_*`` entry point on the current CUDA stream.  None of them
allocates: callers pass every output buffer.
"""
from __future__ import annotations

import torch

from . import _lib
from .partition import UlyssesGeometry


class DeviceStatus:
    """Device int32 status word of the attention kernel plus a lazy host check.

    The kernel writes a non-zero code (PS_B200_DEVICE_TIMEOUT_*) when one of
    its bounded internal waits expires.  ``arm()`` queues a 4-byte copy of the
    word to pinned host memory after a launch; ``poll()`` (cheap, no sync)
    raises if a completed copy shows an error; ``check()`` synchronizes.
    While a CUDA graph is being captured, ``arm`` and ``poll`` do nothing
    (the kernels still write the word; ``check()`` after a replay reads it).
    """

    def __init__(self, device: torch.device):
        self.device = device
        self.word = torch.zeros(1, dtype=torch.int32, device=device)
        self.host = torch.zeros(1, dtype=torch.int32, pin_memory=True)
        self.event = None

    @property
    def ptr(self) -> int:
        return self.word.data_ptr()

    def arm(self):
        if torch.cuda.is_current_stream_capturing():
            return
        self.host.copy_(self.word, non_blocking=True)
        self.event = torch.cuda.Event()
        self.event.record(torch.cuda.current_stream(self.device))

    def poll(self):
        if torch.cuda.is_current_stream_capturing():
            return
        if self.event is not None and self.event.query():
            self._raise_if_set(int(self.host.item()))

    def check(self):
        torch.cuda.current_stream(self.device).synchronize()
        self._raise_if_set(int(self.word.item()))

    def _raise_if_set(self, code: int):
        if code:
            self.word.zero_()
            self.host.zero_()
            raise RuntimeError(f"b200 attention kernel aborted: bounded wait expired (device status {code})")


def _check16(t: torch.Tensor, what: str):
    _lib.require_cuda(t, what)
    if t.dtype not in (torch.bfloat16, torch.float16):
        raise _lib.UnsupportedAttention(f"{what}: bf16/fp16 required, got {t.dtype}")


NORM_NONE, NORM_FULL, NORM_PER_HEAD = 0, 1, 2


def _rope_args(head_dim: int, rope_split_pairs):
    """(style, pairs) for the C ABI: interleaved over the head, or split half."""
    if rope_split_pairs is None:
        return 0, head_dim // 2
    return 1, int(rope_split_pairs)


def _prepass_inputs(x_q, x_k, x_v, w_q, w_k, freqs, geo: UlyssesGeometry, dtype, device, mode: int,
                    rope_split_pairs=None):
    """Validated pointer / stride arguments shared by the two pre-pass entry points."""
    for t, name in ((x_q, "q"), (x_k, "k"), (x_v, "v")):
        _check16(t, f"prepass {name}")
    n = geo.n_local
    width = geo.heads * geo.head_dim
    head_strides = []
    for t, name in ((x_q, "q"), (x_k, "k"), (x_v, "v")):
        if t.dim() == 3 and tuple(t.shape) == (n, geo.heads, geo.head_dim) and t.stride(2) == 1:
            head_strides.append(t.stride(1))
        elif t.dim() == 2 and t.shape[0] == n and t.shape[1] == width and t.stride(1) == 1:
            head_strides.append(geo.head_dim)
        else:
            raise ValueError(f"prepass {name}: expected [{n}, {width}] or [{n}, {geo.heads}, {geo.head_dim}] "
                             f"with unit inner stride, got {tuple(t.shape)} / {t.stride()}")
        if t.dtype != dtype:
            raise ValueError("prepass: q/k/v and exchange dtypes differ")
    w_dtype = _lib.dtype_code(dtype)
    fptr, fstride = 0, 0
    wq = wk = 0
    if mode:
        wlen = width if mode == NORM_FULL else geo.head_dim
        for t, name in ((w_q, "w_q"), (w_k, "w_k")):
            if t.dim() != 1 or t.shape[0] != wlen or not t.is_contiguous() or t.device != device:
                raise ValueError(f"prepass {name}: expected contiguous [{wlen}] on {device}")
        if w_q.dtype != w_k.dtype:
            raise ValueError("prepass: norm weights must share a dtype")
        w_dtype = _lib.dtype_code(w_q.dtype)
        wq, wk = w_q.data_ptr(), w_k.data_ptr()
        if freqs.dtype != torch.float32 or freqs.device != device:
            raise ValueError("prepass: freqs must be fp32 on the exchange device")
        pairs = _rope_args(geo.head_dim, rope_split_pairs)[1]
        if (freqs.dim() != 4 or freqs.shape[0] != n or tuple(freqs.shape[1:]) != (pairs, 2, 2)
                or freqs.stride()[1:] != (4, 2, 1) or freqs.stride(0) % 4 != 0):
            raise ValueError(f"prepass: freqs must be [{n}, {pairs}, 2, 2] with contiguous rows")
        fptr, fstride = freqs.data_ptr(), freqs.stride(0)
    return [x_q.data_ptr(), x_k.data_ptr(), x_v.data_ptr(),
            _lib.i64([x_q.stride(0), x_k.stride(0), x_v.stride(0)]), _lib.i64(head_strides),
            wq, wk, w_dtype, fptr, fstride]


def prepass(x_q, x_k, x_v, w_q, w_k, freqs, send, geo: UlyssesGeometry, eps: float = 1e-6,
            norm_rope=True, rope_split_pairs=None):
    """RMSNorm(q), RMSNorm(k), RoPE, pack into ``send`` [W,3,width,h,D].

    x_*: [n_local, H*D] (row stride may exceed H*D) or [n_local, H, D] with
    any row and head strides (e.g. a [H, L, D] tensor transposed) and unit
    inner stride; freqs: [n_local, D/2, 2, 2] fp32.  norm_rope: False/0 pack
    only, True/1 RMSNorm over the full width (Wan; w_* [H*D]), 2 RMSNorm per
    head (Flux / H3 QK-norm; w_* [D]).  rope_split_pairs: None rotates
    interleaved pairs over the whole head (freqs [n, D/2, 2, 2]); P rotates
    pairs (j, j+P), j < P, and keeps the rest (H3 partial RoPE, freqs
    [n, P, 2, 2]).
    """
    mode = int(norm_rope)
    lib = _lib.load()
    _check16(send, "prepass send")
    if send.dim() == 6:  # batched send buffer [W, 3, B, width, h, D]
        batch = send.shape[2]
        if tuple(send.shape) != geo.send_shape(batch) or not send.is_contiguous():
            raise ValueError(f"prepass: send must be contiguous {geo.send_shape(batch)}")
        prepass_to(x_q, x_k, x_v, w_q, w_k, freqs, send_blocks(send), geo, send.dtype, eps, norm_rope,
                   rope_split_pairs, batch=batch)
        return
    if tuple(send.shape) != geo.send_shape() or not send.is_contiguous():
        raise ValueError(f"prepass: send must be contiguous {geo.send_shape()}")
    args = _prepass_inputs(x_q, x_k, x_v, w_q, w_k, freqs, geo, send.dtype, send.device, mode, rope_split_pairs)
    rc = lib.ps_b200_prepass(
        *args, send.data_ptr(), _lib.dtype_code(send.dtype),
        geo.world, geo.n_local, geo.width, geo.heads, geo.heads_per_rank, geo.head_dim, float(eps),
        mode, *_rope_args(geo.head_dim, rope_split_pairs), _lib.stream_handle(send.device))
    _lib.check(rc, "ps_b200_prepass")


def prepass_to(x_q, x_k, x_v, w_q, w_k, freqs, dst_blocks, geo: UlyssesGeometry, dtype: torch.dtype,
               eps: float = 1e-6, norm_rope=True, rope_split_pairs=None, batch: int | None = None):
    """``prepass`` storing destination d's [3,width,h,D] block at the device
    address ``dst_blocks[d]`` (a peer's receive buffer: the fused exchange).

    With ``batch`` B the inputs carry a leading batch axis (x_* [B, n, H*D]
    or [B, n, H, D], any batch stride; freqs [n, P, 2, 2] shared by the rows
    or [B, n, P, 2, 2]) and each destination block is [3, B, width, h, D]."""
    mode = int(norm_rope)
    lib = _lib.load()
    if len(dst_blocks) != geo.world:
        raise ValueError(f"prepass_to: {len(dst_blocks)} destination blocks for {geo.world} ranks")
    if batch is None:
        args = _prepass_inputs(x_q, x_k, x_v, w_q, w_k, freqs, geo, dtype, x_q.device, mode, rope_split_pairs)
        rc = lib.ps_b200_prepass_to(
            *args, _lib.ptrs(dst_blocks), _lib.dtype_code(dtype),
            geo.world, geo.n_local, geo.width, geo.heads, geo.heads_per_rank, geo.head_dim, float(eps),
            mode, *_rope_args(geo.head_dim, rope_split_pairs), _lib.stream_handle(x_q.device))
        _lib.check(rc, "ps_b200_prepass_to")
        return
    batch = int(batch)
    xs = (x_q, x_k, x_v)
    for t, name in zip(xs, "qkv"):
        if t.dim() not in (3, 4) or t.shape[0] != batch:
            raise ValueError(f"prepass {name}: expected a leading batch axis of {batch}, got {tuple(t.shape)}")
    # Row b of a batched input is x[b]: validate one row, pass the batch strides.
    fb = 0
    f_row = freqs
    if mode and freqs is not None and freqs.dim() == 5:
        if freqs.shape[0] != batch:
            raise ValueError(f"prepass: batched freqs must have {batch} rows")
        fb, f_row = freqs.stride(0), freqs[0]
    args = _prepass_inputs(x_q[0], x_k[0], x_v[0], w_q, w_k, f_row, geo, dtype, x_q.device, mode, rope_split_pairs)
    ptrs = [t.data_ptr() for t in xs]
    rc = lib.ps_b200_prepass_batch(
        *ptrs, _lib.i64([t.stride(0) for t in xs]), *args[3:9], fb, args[9], _lib.ptrs(dst_blocks),
        _lib.dtype_code(dtype), batch, geo.world, geo.n_local, geo.width, geo.heads, geo.heads_per_rank,
        geo.head_dim, float(eps), mode, *_rope_args(geo.head_dim, rope_split_pairs), _lib.stream_handle(x_q.device))
    _lib.check(rc, "ps_b200_prepass_batch")


def send_blocks(send: torch.Tensor):
    """Device address of each destination's block of a local send buffer
    (its slices along the leading world axis)."""
    step = send[0].numel() * send.element_size()
    return [send.data_ptr() + d * step for d in range(send.shape[0])]


def attention_workspace(device: torch.device) -> torch.Tensor:
    """Scratch for the attention entry points (split last wave); one per
    stream of concurrent calls."""
    return torch.empty(_lib.ATTN_WORKSPACE_BYTES, dtype=torch.uint8, device=device)


def _ws(workspace):
    if workspace is None:
        return None, 0
    if workspace.device.type != "cuda" or not workspace.is_contiguous():
        raise ValueError("attention workspace must be a contiguous CUDA tensor")
    return workspace.data_ptr(), workspace.numel() * workspace.element_size()


def _seg_table(geo: UlyssesGeometry):
    """Per-segment row table for the C ABI: None for ceil-width shards."""
    return _lib.i32(geo.sizes) if geo.sizes is not None else None


def ulysses_attention(recv, out_send, geo: UlyssesGeometry, scale: float, status: DeviceStatus | None,
                      workspace=None):
    """Attention over the receive buffer [W,3,width,h,D] for this rank's real heads."""
    lib = _lib.load()
    _check16(recv, "attention recv")
    _lib.require_cuda(out_send, "attention out")
    if recv.dim() == 6:  # batched [W, 3, B, width, h, D] -> out_send [W, B, width, h, D]
        batch = recv.shape[2]
        if tuple(out_send.shape) != geo.out_shape(batch) or not out_send.is_contiguous():
            raise ValueError(f"attention: out must be contiguous {geo.out_shape(batch)}")
        h, d = geo.heads_per_rank, geo.head_dim
        _attention_batch(recv, send_blocks(out_send), geo.width * h * d, h * d, out_send.dtype, geo, batch, scale,
                         status, workspace)
        return
    if tuple(recv.shape) != geo.send_shape() or not recv.is_contiguous():
        raise ValueError(f"attention: recv must be contiguous {geo.send_shape()}")
    if tuple(out_send.shape) != geo.out_shape() or not out_send.is_contiguous():
        raise ValueError(f"attention: out must be contiguous {geo.out_shape()}")
    if out_send.dtype not in (recv.dtype, torch.float32):
        raise ValueError("attention: output dtype must be fp32 or the input dtype")
    rc = lib.ps_b200_ulysses_attn_fwd(
        recv.data_ptr(), out_send.data_ptr(), _lib.dtype_code(recv.dtype), _lib.dtype_code(out_send.dtype),
        geo.world, geo.width, geo.total, _seg_table(geo), geo.heads_per_rank, geo.heads_valid, geo.head_dim,
        float(scale), *_ws(workspace),
        status.ptr if status is not None else None, _lib.stream_handle(recv.device))
    _lib.check(rc, "ps_b200_ulysses_attn_fwd")
    if status is not None:
        status.arm()


def ulysses_joint_attention(recv, prefix_qkv, out_send, prefix_out, geo: UlyssesGeometry, scale: float,
                            status: DeviceStatus | None, workspace=None):
    """Joint attention: this rank's text rows prefix_qkv [3,P,h,D] ahead of the
    image rows of recv [W,3,width,h,D]; text outputs -> prefix_out [P,h,D],
    image outputs -> out_send [W,width,h,D]."""
    lib = _lib.load()
    _check16(recv, "joint attention recv")
    _check16(prefix_qkv, "joint attention prefix")
    if tuple(recv.shape) != geo.send_shape() or not recv.is_contiguous():
        raise ValueError(f"joint attention: recv must be contiguous {geo.send_shape()}")
    h, d = geo.heads_per_rank, geo.head_dim
    if prefix_qkv.dim() != 4 or tuple(prefix_qkv.shape[::2]) != (3, h) or prefix_qkv.shape[3] != d \
            or not prefix_qkv.is_contiguous() or prefix_qkv.dtype != recv.dtype:
        raise ValueError(f"joint attention: prefix must be contiguous [3, P, {h}, {d}]")
    plen = prefix_qkv.shape[1]
    for t, shape, name in ((out_send, geo.out_shape(), "out"), (prefix_out, (plen, h, d), "prefix out")):
        if tuple(t.shape) != tuple(shape) or not t.is_contiguous() or t.dtype not in (recv.dtype, torch.float32):
            raise ValueError(f"joint attention: {name} must be contiguous {tuple(shape)}")
    if out_send.dtype != prefix_out.dtype:
        raise ValueError("joint attention: both outputs need the same dtype")
    rc = lib.ps_b200_ulysses_joint_attn_fwd(
        recv.data_ptr(), prefix_qkv.data_ptr(), out_send.data_ptr(), prefix_out.data_ptr(),
        _lib.dtype_code(recv.dtype), _lib.dtype_code(out_send.dtype), geo.world, geo.width, geo.total, plen,
        _seg_table(geo), h, geo.heads_valid, d, float(scale), *_ws(workspace),
        status.ptr if status is not None else None,
        _lib.stream_handle(recv.device))
    _lib.check(rc, "ps_b200_ulysses_joint_attn_fwd")
    if status is not None:
        status.arm()


def unpack(out_recv, out, geo: UlyssesGeometry):
    """[W,width,h,D] received outputs -> out [n_local, H, D] (real heads only)."""
    lib = _lib.load()
    _check16(out_recv, "unpack recv")
    _lib.require_cuda(out, "unpack out")
    if out_recv.dim() == 5:  # batched [W, B, width, h, D] -> out [B, n, H, D]
        batch = out_recv.shape[1]
        if tuple(out_recv.shape) != geo.out_shape(batch) or not out_recv.is_contiguous():
            raise ValueError(f"unpack: recv must be contiguous {geo.out_shape(batch)}")
        h, d = geo.heads_per_rank, geo.head_dim
        _unpack_batch(out_recv, batch * geo.width * h * d, geo.width * h * d, h * d, out, geo, batch)
        return
    if tuple(out_recv.shape) != geo.out_shape() or not out_recv.is_contiguous():
        raise ValueError(f"unpack: recv must be contiguous {geo.out_shape()}")
    if (out.dim() != 3 or tuple(out.shape) != (geo.n_local, geo.heads, geo.head_dim)
            or out.stride(2) != 1 or out.stride(1) != geo.head_dim):
        raise ValueError(f"unpack: out must be [{geo.n_local}, {geo.heads}, {geo.head_dim}] with packed heads")
    rc = lib.ps_b200_unpack(
        out_recv.data_ptr(), out.data_ptr(), out.stride(0), _lib.dtype_code(out_recv.dtype),
        _lib.dtype_code(out.dtype), geo.world, geo.n_local, geo.width, geo.heads, geo.heads_per_rank,
        geo.head_dim, _lib.stream_handle(out.device))
    _lib.check(rc, "ps_b200_unpack")


def _attention_batch(recv, out_blocks, out_batch_stride: int, out_row_stride: int, out_dtype: torch.dtype,
                     geo: UlyssesGeometry, batch: int, scale: float, status: DeviceStatus | None, workspace=None):
    """Attention over the batched receive buffer [W, 3, B, width, h, D]; batch
    row b, valid row i of segment s, head j -> out_blocks[s] + b*out_batch_stride
    + i*out_row_stride + j*D elements (ps_b200_ulysses_attn_batch)."""
    lib = _lib.load()
    if tuple(recv.shape) != geo.send_shape(batch) or not recv.is_contiguous():
        raise ValueError(f"attention: recv must be contiguous {geo.send_shape(batch)}")
    if len(out_blocks) != geo.world:
        raise ValueError(f"attention: {len(out_blocks)} output blocks for {geo.world} ranks")
    if out_dtype not in (recv.dtype, torch.float32):
        raise ValueError("attention: output dtype must be fp32 or the input dtype")
    rc = lib.ps_b200_ulysses_attn_batch(
        recv.data_ptr(), _lib.ptrs(out_blocks), int(out_batch_stride), int(out_row_stride),
        _lib.dtype_code(recv.dtype), _lib.dtype_code(out_dtype), int(batch), geo.world, geo.width, geo.total,
        _seg_table(geo), geo.heads_per_rank, geo.heads_valid, geo.head_dim, float(scale), *_ws(workspace),
        status.ptr if status is not None else None, _lib.stream_handle(recv.device))
    _lib.check(rc, "ps_b200_ulysses_attn_batch")
    if status is not None:
        status.arm()


def ulysses_attention_to(recv, out_blocks, out_row_stride: int, out_dtype: torch.dtype, geo: UlyssesGeometry,
                         scale: float, status: DeviceStatus | None, workspace=None, batch: int | None = None,
                         out_batch_stride: int = 0):
    """``ulysses_attention`` storing segment s's valid rows at the device
    address ``out_blocks[s]`` (row stride ``out_row_stride`` elements, head j
    at + j*D): each source rank's staging buffer, the fused output exchange.
    With ``batch`` B, recv is [W, 3, B, width, h, D] and batch row b of
    segment s starts at out_blocks[s] + b * out_batch_stride elements."""
    lib = _lib.load()
    _check16(recv, "attention recv")
    if batch is not None:
        _attention_batch(recv, out_blocks, out_batch_stride, out_row_stride, out_dtype, geo, int(batch), scale,
                         status, workspace)
        return
    if tuple(recv.shape) != geo.send_shape() or not recv.is_contiguous():
        raise ValueError(f"attention: recv must be contiguous {geo.send_shape()}")
    if len(out_blocks) != geo.world:
        raise ValueError(f"attention: {len(out_blocks)} output blocks for {geo.world} ranks")
    if out_dtype not in (recv.dtype, torch.float32):
        raise ValueError("attention: output dtype must be fp32 or the input dtype")
    rc = lib.ps_b200_ulysses_attn_to(
        recv.data_ptr(), _lib.ptrs(out_blocks), int(out_row_stride), _lib.dtype_code(recv.dtype),
        _lib.dtype_code(out_dtype), geo.world, geo.width, geo.total, _seg_table(geo), geo.heads_per_rank,
        geo.heads_valid, geo.head_dim, float(scale), *_ws(workspace), status.ptr if status is not None else None,
        _lib.stream_handle(recv.device))
    _lib.check(rc, "ps_b200_ulysses_attn_to")
    if status is not None:
        status.arm()


def ulysses_joint_attention_to(recv, prefix_qkv, out_blocks, out_row_stride: int, prefix_out,
                               out_dtype: torch.dtype, geo: UlyssesGeometry, scale: float,
                               status: DeviceStatus | None, workspace=None):
    """``ulysses_joint_attention`` with the image outputs stored through one
    device address per source segment (the owners' staging buffers)."""
    lib = _lib.load()
    _check16(recv, "joint attention recv")
    _check16(prefix_qkv, "joint attention prefix")
    if tuple(recv.shape) != geo.send_shape() or not recv.is_contiguous():
        raise ValueError(f"joint attention: recv must be contiguous {geo.send_shape()}")
    h, d = geo.heads_per_rank, geo.head_dim
    if prefix_qkv.dim() != 4 or tuple(prefix_qkv.shape[::2]) != (3, h) or prefix_qkv.shape[3] != d \
            or not prefix_qkv.is_contiguous() or prefix_qkv.dtype != recv.dtype:
        raise ValueError(f"joint attention: prefix must be contiguous [3, P, {h}, {d}]")
    plen = prefix_qkv.shape[1]
    if tuple(prefix_out.shape) != (plen, h, d) or not prefix_out.is_contiguous() or prefix_out.dtype != out_dtype:
        raise ValueError(f"joint attention: prefix out must be contiguous [{plen}, {h}, {d}] {out_dtype}")
    if len(out_blocks) != geo.world:
        raise ValueError(f"joint attention: {len(out_blocks)} output blocks for {geo.world} ranks")
    rc = lib.ps_b200_ulysses_joint_attn_to(
        recv.data_ptr(), prefix_qkv.data_ptr(), _lib.ptrs(out_blocks), int(out_row_stride), prefix_out.data_ptr(),
        _lib.dtype_code(recv.dtype), _lib.dtype_code(out_dtype), geo.world, geo.width, geo.total, plen,
        _seg_table(geo), h, geo.heads_valid, d, float(scale), *_ws(workspace),
        status.ptr if status is not None else None, _lib.stream_handle(recv.device))
    _lib.check(rc, "ps_b200_ulysses_joint_attn_to")
    if status is not None:
        status.arm()


def broadcast(dst_ptrs, src: torch.Tensor):
    """Copy the contiguous tensor ``src`` to every device address of
    ``dst_ptrs`` (this GPU's memory or peers')."""
    lib = _lib.load()
    _lib.require_cuda(src, "broadcast")
    if not src.is_contiguous():
        raise ValueError("broadcast: source must be contiguous")
    rc = lib.ps_b200_broadcast(_lib.ptrs(dst_ptrs), len(dst_ptrs), src.data_ptr(), src.numel() * src.element_size(),
                               _lib.stream_handle(src.device))
    _lib.check(rc, "ps_b200_broadcast")


def _unpack_batch(src, src_stride: int, batch_stride: int, row_stride: int, out, geo: UlyssesGeometry, batch: int):
    """Head blocks of ``src`` (block s, batch row b, token i at src + s*src_stride
    + b*batch_stride + i*row_stride elements) -> out [B, n_local, H, D]."""
    lib = _lib.load()
    if (out.dim() != 4 or tuple(out.shape) != (batch, geo.n_local, geo.heads, geo.head_dim)
            or out.stride(3) != 1 or out.stride(2) != geo.head_dim):
        raise ValueError(f"unpack: out must be [{batch}, {geo.n_local}, {geo.heads}, {geo.head_dim}] "
                         "with packed heads")
    rc = lib.ps_b200_unpack_batch(
        src.data_ptr(), int(src_stride), int(batch_stride), int(row_stride), out.data_ptr(), out.stride(0),
        out.stride(1), _lib.dtype_code(src.dtype), _lib.dtype_code(out.dtype), int(batch), geo.n_local, geo.heads,
        geo.heads_per_rank, geo.head_dim, _lib.stream_handle(out.device))
    _lib.check(rc, "ps_b200_unpack_batch")


def unpack_staged(staging, out, geo: UlyssesGeometry):
    """Staging buffer [width, W*h, D] (rows of this rank, every head block) ->
    out [n_local, H, D] (real heads only)."""
    lib = _lib.load()
    _check16(staging, "unpack staging")
    _lib.require_cuda(out, "unpack out")
    if staging.dim() == 4:  # batched [B, width, W*h, D] -> out [B, n, H, D]
        batch = staging.shape[0]
        shape = (batch, geo.width, geo.padded_heads, geo.head_dim)
        if tuple(staging.shape) != shape or not staging.is_contiguous():
            raise ValueError(f"unpack: staging must be contiguous {shape}")
        h, d = geo.heads_per_rank, geo.head_dim
        _unpack_batch(staging, h * d, geo.width * geo.padded_heads * d, geo.padded_heads * d, out, geo, batch)
        return
    shape = (geo.width, geo.padded_heads, geo.head_dim)
    if tuple(staging.shape) != shape or not staging.is_contiguous():
        raise ValueError(f"unpack: staging must be contiguous {shape}")
    if (out.dim() != 3 or tuple(out.shape) != (geo.n_local, geo.heads, geo.head_dim)
            or out.stride(2) != 1 or out.stride(1) != geo.head_dim):
        raise ValueError(f"unpack: out must be [{geo.n_local}, {geo.heads}, {geo.head_dim}] with packed heads")
    h, d = geo.heads_per_rank, geo.head_dim
    rc = lib.ps_b200_unpack_strided(
        staging.data_ptr(), h * d, geo.padded_heads * d, out.data_ptr(), out.stride(0),
        _lib.dtype_code(staging.dtype), _lib.dtype_code(out.dtype), geo.n_local, geo.heads, h, d,
        _lib.stream_handle(out.device))
    _lib.check(rc, "ps_b200_unpack_strided")


def token_pack(x_q, x_k, x_v, w_q, w_k, freqs, qkv, n_local: int, heads: int, head_dim: int, eps: float = 1e-6,
               norm_rope=True, rope_split_pairs=None):
    """Token mode, step 1: RMSNorm + RoPE of this rank's rows into the local
    block ``qkv`` [3, width, H, D] (all heads; rows n_local..width-1 zero),
    whose k/v part [2, width, H, D] is what the all-gather moves."""
    mode = int(norm_rope)
    lib = _lib.load()
    _check16(qkv, "token pack")
    width = qkv.shape[1]
    if qkv.dim() != 4 or tuple(qkv.shape) != (3, width, heads, head_dim) or not qkv.is_contiguous():
        raise ValueError(f"token pack: qkv must be contiguous [3, width, {heads}, {head_dim}]")
    geo = UlyssesGeometry(total=n_local, heads=heads, head_dim=head_dim, world=1, rank=0)
    args = _prepass_inputs(x_q, x_k, x_v, w_q, w_k, freqs, geo, qkv.dtype, qkv.device, mode, rope_split_pairs)
    rc = lib.ps_b200_prepass(
        *args, qkv.data_ptr(), _lib.dtype_code(qkv.dtype), 1, n_local, width, heads, heads, head_dim,
        float(eps), mode, *_rope_args(head_dim, rope_split_pairs), _lib.stream_handle(qkv.device))
    _lib.check(rc, "ps_b200_prepass (token mode)")


def token_pack_to(x_q, x_k, x_v, w_q, w_k, freqs, q_out, kv_dst, n_local: int, heads: int, head_dim: int,
                  eps: float = 1e-6, norm_rope=True, rope_split_pairs=None):
    """Token mode with the K/V all-gather as stores: q of this rank's rows to
    ``q_out`` [width, H, D], k/v to the [2, width, H, D] block at each device
    address of ``kv_dst`` (every rank's gathered K/V, this rank's slot)."""
    mode = int(norm_rope)
    lib = _lib.load()
    _check16(q_out, "token pack q")
    width = q_out.shape[0]
    if q_out.dim() != 3 or tuple(q_out.shape[1:]) != (heads, head_dim) or not q_out.is_contiguous():
        raise ValueError(f"token pack: q_out must be contiguous [width, {heads}, {head_dim}]")
    geo = UlyssesGeometry(total=n_local, heads=heads, head_dim=head_dim, world=1, rank=0)
    args = _prepass_inputs(x_q, x_k, x_v, w_q, w_k, freqs, geo, q_out.dtype, q_out.device, mode, rope_split_pairs)
    rc = lib.ps_b200_prepass_token_to(
        *args, q_out.data_ptr(), _lib.ptrs(kv_dst), len(kv_dst), _lib.dtype_code(q_out.dtype), n_local, width,
        heads, head_dim, float(eps), mode, *_rope_args(head_dim, rope_split_pairs), _lib.stream_handle(q_out.device))
    _lib.check(rc, "ps_b200_prepass_token_to")


def token_attention(q, kv_all, out, n_local: int, total: int, scale: float, status: DeviceStatus | None,
                    workspace=None):
    """Token mode, step 3: this rank's queries q [width, H, D] (first n_local
    rows; a [3, width, H, D] block is read as its q part) against the gathered
    keys/values kv_all [W, 2, width, H, D] (segment s holds rank s's
    shard_bounds rows) -> out [n_local, H, D] directly."""
    lib = _lib.load()
    if q.dim() == 4:
        q = q[0]
    _check16(q, "token attention q")
    _check16(kv_all, "token attention kv")
    _lib.require_cuda(out, "token attention out")
    if not q.is_contiguous():
        raise ValueError("token attention: q must be contiguous")
    width, heads, d = q.shape
    world = kv_all.shape[0]
    if tuple(kv_all.shape) != (world, 2, width, heads, d) or not kv_all.is_contiguous():
        raise ValueError(f"token attention: kv_all must be contiguous [W, 2, {width}, {heads}, {d}]")
    if tuple(out.shape) != (n_local, heads, d) or not out.is_contiguous() or out.dtype not in (q.dtype,
                                                                                            torch.float32):
        raise ValueError(f"token attention: out must be contiguous [{n_local}, {heads}, {d}]")
    row, seg = heads * d, 2 * width * heads * d
    q_st = _lib.i64([0, 0, row, d])
    kv_st = _lib.i64([0, seg, row, d])
    o_st = _lib.i64([0, 0, row, d])
    esize = kv_all.element_size()
    rc = lib.ps_b200_attn_fwd(
        q.data_ptr(), q_st, kv_all.data_ptr(), kv_st, kv_all.data_ptr() + width * row * esize, kv_st,
        out.data_ptr(), o_st, _lib.dtype_code(q.dtype), _lib.dtype_code(out.dtype), 1, heads, heads, d,
        width, 1, n_local, width, world, total, float(scale), *_ws(workspace),
        status.ptr if status is not None else None, _lib.stream_handle(q.device))
    _lib.check(rc, "ps_b200_attn_fwd (token mode)")
    if status is not None:
        status.arm()


def attention_blhd(q, k, v, out, scale: float, status: DeviceStatus | None, workspace=None):
    """softmax(Q K^T * scale) V for BLHD tensors (GQA by head grouping)."""
    lib = _lib.load()
    for t, name in ((q, "q"), (k, "k"), (v, "v")):
        _check16(t, f"attention {name}")
        if t.stride(3) != 1:
            raise ValueError(f"attention {name}: head_dim must be contiguous")
    _lib.require_cuda(out, "attention out")
    b, lq, hq, d = q.shape
    lk, hk = k.shape[1], k.shape[2]

    def st(t):  # {batch, segment, row, head}; one segment spanning the sequence
        return _lib.i64([t.stride(0), t.stride(0), t.stride(1), t.stride(2)])

    rc = lib.ps_b200_attn_fwd(
        q.data_ptr(), st(q), k.data_ptr(), st(k), v.data_ptr(), st(v), out.data_ptr(), st(out),
        _lib.dtype_code(q.dtype), _lib.dtype_code(out.dtype), b, hq, hk, d,
        lq, 1, lq, lk, 1, lk, float(scale), *_ws(workspace), status.ptr if status is not None else None,
        _lib.stream_handle(q.device))
    _lib.check(rc, "ps_b200_attn_fwd")
    if status is not None:
        status.arm()


# ------------------------------------------------------------ projection GEMMs
def projection_workspace(rows: int, heads: int, head_dim: int, device: torch.device) -> torch.Tensor:
    """Scratch of ``qkv_projection`` for ``rows`` = batch * n_local rows (per-row
    partial sums of squares and group counters); one per stream of
    concurrent calls."""
    lib = _lib.load()
    nbytes = int(lib.ps_b200_qkv_proj_workspace_bytes(int(rows), int(heads), int(head_dim)))
    return torch.empty(max(nbytes, 16), dtype=torch.uint8, device=device)


def _opt_ptr(t):
    return None if t is None else t.data_ptr()


def _vector(t, n, name, device):
    if t is None:
        return None
    if t.dim() != 1 or t.shape[0] != n or not t.is_contiguous() or t.device != device:
        raise ValueError(f"{name}: expected a contiguous [{n}] tensor on {device}")
    return t


def qkv_projection(x, w_q, w_k, w_v, b_q, b_k, b_v, norm_q, norm_k, freqs, dst_blocks, geo: UlyssesGeometry,
                   eps: float, workspace: torch.Tensor, status: DeviceStatus | None = None):
    """q|k|v = x W^T + b with RMSNorm (full width), norm weights and RoPE on q/k,
    stored straight into destination d's block at the device address
    ``dst_blocks[d]`` (a slice of the local send buffer or a peer's receive
    buffer) - the projections plus the whole pre-pass in one kernel.

    x [n_local, in_features], or [B, n_local, in_features] for a batch of
    rows in one GEMM (destination blocks [3, B, width, h, D]); unit inner
    stride, batch rows one after the other.  w_* [H*D, in_features]
    contiguous (PyTorch Linear weights, x's dtype), b_* [H*D] or None,
    norm_* [H*D] (fp32 or x's dtype), freqs [n_local, D/2, 2, 2] fp32 (or
    [B, n_local, D/2, 2, 2]).  workspace: ``projection_workspace(B * n_local, ...)``."""
    lib = _lib.load()
    _check16(x, "projection x")
    device, dtype = x.device, x.dtype
    width = geo.heads * geo.head_dim
    batch = x.shape[0] if x.dim() == 3 else 1
    rows = x if x.dim() == 2 else x.reshape(batch * x.shape[1], x.shape[2])
    if rows.shape[0] != batch * geo.n_local or rows.stride(-1) != 1 or (x.dim() == 3 and x.shape[1] != geo.n_local):
        raise ValueError(f"projection x: expected [{geo.n_local}, in_features] or [B, {geo.n_local}, in_features] "
                         "with unit inner stride and consecutive batch rows")
    if x.dim() == 3 and batch > 1 and x.stride(0) != geo.n_local * x.stride(1):
        raise ValueError("projection x: batch rows must follow each other")
    fin = rows.shape[1]
    for t, name in ((w_q, "w_q"), (w_k, "w_k"), (w_v, "w_v")):
        if t.dtype != dtype or tuple(t.shape) != (width, fin) or not t.is_contiguous() or t.device != device:
            raise ValueError(f"projection {name}: expected contiguous [{width}, {fin}] {dtype}")
    biases = [_vector(b, width, f"b_{n}", device) for b, n in ((b_q, "q"), (b_k, "k"), (b_v, "v"))]
    bdt = next((b.dtype for b in biases if b is not None), torch.float32)
    if any(b is not None and b.dtype != bdt for b in biases):
        raise ValueError("projection biases must share a dtype")
    _vector(norm_q, width, "norm_q", device)
    _vector(norm_k, width, "norm_k", device)
    if norm_q.dtype != norm_k.dtype:
        raise ValueError("projection norm weights must share a dtype")
    fb = 0
    table = freqs
    if freqs.dim() == 5:
        if freqs.shape[0] != batch:
            raise ValueError(f"projection freqs: {freqs.shape[0]} tables for {batch} batch rows")
        fb, table = freqs.stride(0), freqs[0]
    if (table.dtype != torch.float32 or table.dim() != 4 or table.shape[0] != geo.n_local
            or tuple(table.shape[1:]) != (geo.head_dim // 2, 2, 2) or table.stride()[1:] != (4, 2, 1)):
        raise ValueError(f"projection freqs: expected [{geo.n_local}, {geo.head_dim // 2}, 2, 2] fp32")
    if len(dst_blocks) != geo.world:
        raise ValueError(f"projection: {len(dst_blocks)} destination blocks for {geo.world} ranks")
    rc = lib.ps_b200_qkv_proj_batch(
        rows.data_ptr(), rows.stride(0), w_q.data_ptr(), w_k.data_ptr(), w_v.data_ptr(),
        *[_opt_ptr(b) for b in biases], _lib.dtype_code(bdt), norm_q.data_ptr(), norm_k.data_ptr(),
        _lib.dtype_code(norm_q.dtype), table.data_ptr(), fb, table.stride(0), _lib.ptrs(dst_blocks),
        _lib.dtype_code(dtype), batch, geo.world, geo.n_local, geo.width, geo.heads, geo.heads_per_rank,
        geo.head_dim, fin, float(eps), *_ws(workspace), status.ptr if status is not None else None,
        _lib.stream_handle(device))
    _lib.check(rc, "ps_b200_qkv_proj_batch")
    if status is not None:
        status.arm()


def out_projection(src, w_o, b_o, out, n_local: int, in_features: int, row_stride: int, block_stride: int = 0,
                   block_cols: int = 0, status: DeviceStatus | None = None):
    """out = A W_o^T + b_o with A row i read in place from ``src`` (a tensor or
    its storage): row i at element i*row_stride, or - with block_cols > 0 -
    its columns [b*block_cols, (b+1)*block_cols) at b*block_stride +
    i*row_stride (the NCCL receive buffer's per-source blocks)."""
    lib = _lib.load()
    _check16(src, "projection source")
    _lib.require_cuda(out, "projection out")
    dtype = src.dtype
    fout = w_o.shape[0]
    if w_o.dtype != dtype or tuple(w_o.shape) != (fout, in_features) or not w_o.is_contiguous():
        raise ValueError(f"projection w_o: expected contiguous [out_features, {in_features}] {dtype}")
    b_o = _vector(b_o, fout, "b_o", src.device)
    if out.dim() != 2 or tuple(out.shape) != (n_local, fout) or out.stride(1) != 1 or out.dtype not in (
            dtype, torch.float32):
        raise ValueError(f"projection out: expected [{n_local}, {fout}] with unit inner stride")
    rc = lib.ps_b200_out_proj(
        src.data_ptr(), int(row_stride), int(block_stride), int(block_cols), w_o.data_ptr(), _opt_ptr(b_o),
        _lib.dtype_code(b_o.dtype if b_o is not None else torch.float32), out.data_ptr(), out.stride(0),
        _lib.dtype_code(dtype), _lib.dtype_code(out.dtype), int(n_local), int(in_features), int(fout),
        status.ptr if status is not None else None, _lib.stream_handle(src.device))
    _lib.check(rc, "ps_b200_out_proj")
    if status is not None:
        status.arm()
