"""Ulysses sequence-parallel self-attention of one block on this rank.

Data path (one process per GPU, NCCL through torch.distributed):

  pre-pass kernel   q/k RMSNorm + RoPE, written straight into the send buffer
                    send [W][3][width][h][D] (bf16)
  all_to_all_single send -> recv (skipped when W == 1: recv is send)
  attention kernel  reads recv in place (one key/value segment per source
                    rank) for this rank's h heads, writes the output send
                    buffer [W][width][h][D] - or, when W == 1, the final
                    [n][H][D] output directly
  all_to_all_single out_send -> out_recv
  unpack kernel     out_recv -> [n][H][D], dropping padded heads

With the peer exchange (one node, NVLink; ``exchange="auto"|"peer"``) the
two all_to_all_single calls disappear: the pre-pass stores each
destination's block straight into that rank's receive buffer, the attention
epilogue stores each output row straight into its owner's staging buffer,
and two 4-byte all-reduces order the steps across ranks (``peer.py``).

This replaces powershard/wan_model.py:421-430 (attention_qkv) + 343-364
(ulysses_to_sequence) + 398-418 (run_attention) + 367-381
(ulysses_to_heads) for a whole batch (e.g. the CFG pair) in one exchange,
with the reference's batched packing [W][3][B][width][h][D].  Buffers are
cached per (device, stream, geometry, batch, dtype) and reused; the
returned output is always a fresh tensor.
"""
from __future__ import annotations

import contextlib

import torch
import torch.distributed as dist

from . import ops
from .partition import UlyssesGeometry, shard_bounds


class UlyssesAttention:
    """Per-rank engine; `group` is the sequence-parallel process group.

    ``kernels`` is the set of device steps (default: the CUDA kernels of
    ``ops``: ``prepass``, ``ulysses_attention``, ``unpack``, ``DeviceStatus``
    with the same buffer contracts).  Only tests replace it, to exercise the
    exchange logic over CPU collectives; CPU tensors given to the default
    kernels raise.

    ``exchange`` picks how q/k/v and outputs cross ranks: ``"nccl"`` - two
    ``all_to_all_single`` calls per block, as the reference; ``"peer"`` - the
    kernels store straight into the other ranks' buffers over NVLink
    (``peer.PeerExchange``; raises if the ranks cannot map each other's
    memory); ``"auto"`` (default) - peer when the group is NCCL on one node
    and every rank can map its peers, else nccl.
    """

    def __init__(self, group=None, kernels=None, exchange: str = "auto"):
        if exchange not in ("auto", "nccl", "peer"):
            raise ValueError(f"exchange must be auto, nccl or peer, not {exchange!r}")
        self.group = group
        self.kernels = kernels if kernels is not None else ops
        self.exchange = exchange
        self._buffers = {}
        self._status = {}
        self._peers = {}
        self._attn_ws = {}
        self.last_exchange = None  # exchange the last token-mode call used

    # ------------------------------------------------------------ topology
    def world_rank(self):
        if dist.is_available() and dist.is_initialized():
            return dist.get_world_size(self.group), dist.get_rank(self.group)
        return 1, 0

    def geometry(self, total: int, heads: int, head_dim: int, local: bool = False,
                 sizes=None) -> UlyssesGeometry:
        world, rank = (1, 0) if local else self.world_rank()
        if sizes is not None and len(sizes) != world:
            raise ValueError(f"{len(sizes)} split sizes for a group of {world} ranks")
        return UlyssesGeometry(total=total, heads=heads, head_dim=head_dim, world=world, rank=rank,
                               sizes=None if sizes is None else tuple(sizes))

    # ------------------------------------------------------------ buffers
    def _workspace(self, geo: UlyssesGeometry, dtype: torch.dtype, device: torch.device, batch: int | None = None):
        stream = torch.cuda.current_stream(device).cuda_stream if device.type == "cuda" else 0
        key = (device.index, stream, geo.world, geo.width, geo.heads_per_rank, geo.head_dim, dtype, batch)
        ws = self._buffers.get(key)
        if ws is None:
            send = torch.empty(geo.send_shape(batch), dtype=dtype, device=device)
            recv = send if geo.world == 1 else torch.empty_like(send)
            out_send = None if geo.world == 1 else torch.empty(geo.out_shape(batch), dtype=dtype, device=device)
            out_recv = None if geo.world == 1 else torch.empty_like(out_send)
            ws = dict(send=send, recv=recv, out_send=out_send, out_recv=out_recv)
            self._buffers[key] = ws
        return ws, self._device_status(device)

    def _exchange(self, recv, send, geo):
        if geo.world > 1:
            dist.all_to_all_single(recv, send, group=self.group)

    def _peer(self, geo: UlyssesGeometry, dtype: torch.dtype, device: torch.device, text_rows: int = 0,
              layout: str = "ulysses", batch: int | None = None):
        """The peer exchange of this geometry, or None for the NCCL path."""
        if geo.world == 1 or self.exchange == "nccl" or self.kernels is not ops or device.type != "cuda":
            return None
        if self.exchange == "auto" and dist.get_backend(self.group) != "nccl":
            return None
        stream = torch.cuda.current_stream(device).cuda_stream
        key = (layout, device.index, stream, geo.world, geo.rank, geo.width, geo.heads, geo.head_dim, dtype,
               text_rows, batch)
        if key not in self._peers:
            from .peer import PeerExchange
            ex = PeerExchange.create(self.group, geo, dtype, device, text_rows, layout, batch)
            if ex is None and self.exchange == "peer":
                raise RuntimeError("peer exchange requested but the ranks cannot map each other's memory")
            self._peers[key] = ex
        return self._peers[key]

    def close(self):
        """Release peer-exchange buffers (collective: call on every rank)."""
        for ex in self._peers.values():
            if ex is not None:
                ex.close()
        self._peers.clear()

    # ------------------------------------------------------------ forward
    def forward(self, x_q, x_k, x_v, w_q=None, w_k=None, freqs=None, *, total: int, heads: int,
                eps: float = 1e-6, scale: float | None = None, out_dtype: torch.dtype | None = None,
                norm_rope: bool = True, state: dict | None = None, local: bool = False,
                rope_split_pairs: int | None = None) -> torch.Tensor:
        """One block's self-attention for this rank's tokens (one batch row).

        x_q/x_k/x_v: [n_local, H*D] (or [n_local, H, D]) q/k/v projection
        outputs (bf16/fp16).  With norm_rope, w_q/w_k [H*D] are the RMSNorm
        weights and freqs is the rank's rotation table [n_local, D/2, 2, 2]
        fp32; without it the inputs are already normalised/rotated and are
        only exchanged.  norm_rope may also be ops.NORM_PER_HEAD (w_q/w_k
        [D]); rope_split_pairs P selects the split-half partial RoPE of H3
        (freqs [n_local, P, 2, 2]).  Returns [n_local, H, D] in out_dtype
        (default: the input dtype).  local=True runs the block on this rank
        alone (no exchange, W = 1).  ``forward_batch`` is the same for a
        batch of rows in one exchange.
        """
        return self.forward_batch(x_q[None], x_k[None], x_v[None], w_q, w_k, freqs, total=total, heads=heads,
                                  eps=eps, scale=scale, out_dtype=out_dtype, norm_rope=norm_rope, state=state,
                                  local=local, rope_split_pairs=rope_split_pairs)[0]

    def forward_batch(self, x_q, x_k, x_v, w_q=None, w_k=None, freqs=None, *, total: int, heads: int,
                      eps: float = 1e-6, scale: float | None = None, out_dtype: torch.dtype | None = None,
                      norm_rope: bool = True, state: dict | None = None, local: bool = False,
                      rope_split_pairs: int | None = None) -> torch.Tensor:
        """``forward`` for B batch rows in one exchange, as the reference
        moves a whole batch with one all_to_all_single each way
        (powershard/wan_model.py:356-362, :373-378).

        x_*: [B, n_local, H*D] or [B, n_local, H, D] (any batch/row/head
        strides, unit inner stride); freqs [n_local, P, 2, 2] shared by the
        rows, or [B, n_local, P, 2, 2].  Returns [B, n_local, H, D].  One
        pre-pass, one attention launch and one unpack serve the whole batch;
        the state counters count the batch's bytes once.
        """
        device = x_q.device
        dtype = x_q.dtype
        batch = x_q.shape[0]
        head_dim = x_q.shape[-1] if x_q.dim() == 4 else x_q.shape[-1] // heads
        geo = self.geometry(total, heads, head_dim, local)
        if x_q.shape[1] != geo.n_local:
            raise ValueError("Ulysses local token/head geometry mismatch")
        out_dtype = out_dtype or dtype
        scale = head_dim ** -0.5 if scale is None else float(scale)
        k = self.kernels
        h, d = geo.heads_per_rank, head_dim
        with torch.cuda.device(device) if device.type == "cuda" else contextlib.nullcontext():
            out = torch.empty((batch, geo.n_local, heads, head_dim), dtype=out_dtype, device=device)
            if batch == 0:
                return out
            px = self._peer(geo, dtype, device, batch=batch)
            if px is not None:
                status = self._device_status(device)
                status.poll()
                k.prepass_to(x_q, x_k, x_v, w_q, w_k, freqs, px.dst_blocks, geo, dtype, eps, norm_rope,
                             **self._rope_kw(rope_split_pairs), batch=batch)
                px.barrier()
                k.ulysses_attention_to(px.recv, px.out_blocks, px.out_row_stride, dtype, geo, scale, status,
                                       **self._ws(device), batch=batch, out_batch_stride=px.out_batch_stride)
                px.barrier()
                k.unpack_staged(px.staging, out, geo)
                self._count(state, geo, dtype, "peer", batch)
                return out
            ws, status = self._workspace(geo, dtype, device, batch)
            status.poll()
            k.prepass(x_q, x_k, x_v, w_q, w_k, freqs, ws["send"], geo, eps, norm_rope,
                      **self._rope_kw(rope_split_pairs))
            self._exchange(ws["recv"], ws["send"], geo)
            if geo.world == 1:
                # The final [B, n, H, D] output is the only segment's output block.
                k.ulysses_attention(ws["recv"], out.view(1, batch, geo.n_local, heads, head_dim), geo, scale,
                                    status, **self._ws(device))
            else:
                k.ulysses_attention(ws["recv"], ws["out_send"], geo, scale, status, **self._ws(device))
                self._exchange(ws["out_recv"], ws["out_send"], geo)
                k.unpack(ws["out_recv"], out, geo)
        self._count(state, geo, dtype, "nccl" if geo.world > 1 else "local", batch)
        return out

    def forward_layer(self, x, w_q, w_k, w_v, w_o, norm_q, norm_k, freqs, b_q=None, b_k=None, b_v=None, b_o=None,
                      *, total: int, heads: int, eps: float = 1e-6, scale: float | None = None,
                      out_dtype: torch.dtype | None = None, state: dict | None = None,
                      local: bool = False) -> torch.Tensor:
        """The whole self-attention layer of this rank's tokens in the fused
        kernels: [B, n_local, in_features] -> [B, n_local, out_features].

        The q/k/v projections, RMSNorm over the full width, RoPE and the
        Ulysses pack run as one GEMM (``ps_b200_qkv_proj_batch``) whose
        epilogue stores into the send layout or the peers' receive buffers;
        then the exchange, attention and the inverse exchange as in
        ``forward_batch``; the output projection (``ps_b200_out_proj``) reads
        the attention output from the exchange buffer in place.  So neither
        the projections nor the attention output make a separate round trip
        through HBM (powershard/wan_model.py:425-438 in one pass).

        x and the weights share the 16-bit wire type (w_* [H*D, in_features],
        w_o [out_features, H*D], PyTorch Linear layout); biases [*] or None;
        norm_* [H*D]; freqs [n_local, D/2, 2, 2] fp32 (or one table per batch
        row).  Needs the CUDA kernels (head_dim 128, an even head count).
        """
        if self.kernels is not ops or x.device.type != "cuda":
            raise RuntimeError("forward_layer runs on the CUDA kernels only")
        device, dtype = x.device, x.dtype
        batch, n, _ = x.shape
        head_dim = w_q.shape[0] // heads
        geo = self.geometry(total, heads, head_dim, local)
        if n != geo.n_local:
            raise ValueError("Ulysses local token/head geometry mismatch")
        out_dtype = out_dtype or dtype
        scale = head_dim ** -0.5 if scale is None else float(scale)
        fout = w_o.shape[0]
        hd = heads * head_dim
        h = geo.heads_per_rank
        out = torch.empty((batch, n, fout), dtype=out_dtype, device=device)
        if batch == 0:
            return out
        x = x if x.is_contiguous() else x.contiguous()
        with torch.cuda.device(device):
            status = self._device_status(device)
            status.poll()
            pws = self._proj_workspace(device, batch * n, heads, head_dim)
            px = self._peer(geo, dtype, device, batch=batch)
            if px is not None:
                ops.qkv_projection(x, w_q, w_k, w_v, b_q, b_k, b_v, norm_q, norm_k, freqs, px.dst_blocks, geo, eps,
                                   pws, status)
                px.barrier()
                ops.ulysses_attention_to(px.recv, px.out_blocks, px.out_row_stride, dtype, geo, scale, status,
                                         **self._ws(device), batch=batch, out_batch_stride=px.out_batch_stride)
                px.barrier()
                for b in range(batch):  # staging rows [width][W*h][D]: the first H*D columns in head order
                    ops.out_projection(px.staging[b], w_o, b_o, out[b], n, hd, geo.padded_heads * head_dim,
                                       status=status)
                self._count(state, geo, dtype, "peer", batch)
                return out
            ws, _ = self._workspace(geo, dtype, device, batch)
            ops.qkv_projection(x, w_q, w_k, w_v, b_q, b_k, b_v, norm_q, norm_k, freqs, ops.send_blocks(ws["send"]),
                               geo, eps, pws, status)
            self._exchange(ws["recv"], ws["send"], geo)
            if geo.world == 1:
                key = ("attn_out", device.index, torch.cuda.current_stream(device).cuda_stream, batch, n, hd, dtype)
                attn = self._buffers.get(key)
                if attn is None:
                    attn = self._buffers[key] = torch.empty((batch, n, heads, head_dim), dtype=dtype, device=device)
                ops.ulysses_attention(ws["recv"], attn.view(1, batch, n, heads, head_dim), geo, scale, status,
                                      **self._ws(device))
                for b in range(batch):
                    ops.out_projection(attn[b], w_o, b_o, out[b], n, hd, hd, status=status)
            else:
                ops.ulysses_attention(ws["recv"], ws["out_send"], geo, scale, status, **self._ws(device))
                self._exchange(ws["out_recv"], ws["out_send"], geo)
                for b in range(batch):  # receive blocks [W][B][width][h][D]: heads of source s in block s
                    ops.out_projection(ws["out_recv"][0, b], w_o, b_o, out[b], n, hd, h * head_dim,
                                       block_stride=batch * geo.width * h * head_dim, block_cols=h * head_dim,
                                       status=status)
        self._count(state, geo, dtype, "nccl" if geo.world > 1 else "local", batch)
        return out

    def _proj_workspace(self, device, rows: int, heads: int, head_dim: int):
        key = ("proj_ws", device.index, torch.cuda.current_stream(device).cuda_stream, rows, heads, head_dim)
        ws = self._buffers.get(key)
        if ws is None:
            ws = self._buffers[key] = ops.projection_workspace(rows, heads, head_dim, device)
        return ws

    def _ws(self, device) -> dict:
        """Keyword argument with the attention workspace of (device, stream)
        for the CUDA kernels; stand-in kernels take none."""
        if self.kernels is not ops or device.type != "cuda":
            return {}
        key = (device.index, torch.cuda.current_stream(device).cuda_stream)
        if key not in self._attn_ws:
            self._attn_ws[key] = ops.attention_workspace(device)
        return {"workspace": self._attn_ws[key]}

    @staticmethod
    def _rope_kw(rope_split_pairs) -> dict:
        return {} if rope_split_pairs is None else {"rope_split_pairs": rope_split_pairs}

    def _device_status(self, device):
        if device.index not in self._status:
            self._status[device.index] = self.kernels.DeviceStatus(device)
        return self._status[device.index]

    @staticmethod
    def _count(state, geo, dtype, exchange, batch=1):
        """The reference's sequence-state counters (powershard/wan_model.py:441-502):
        one q/k/v exchange and one output exchange per block, with the bytes
        of the whole batch's send buffers (wan_model.py:364, :381)."""
        if state is None:
            return
        qkv_bytes, out_bytes = geo.exchanged_bytes(dtype.itemsize, batch)
        state["padded_heads"] = geo.padded_heads
        state["kv_collectives"] = state.get("kv_collectives", 0) + 1
        state["kv_gathered_bytes"] = state.get("kv_gathered_bytes", 0) + qkv_bytes
        state["out_collectives"] = state.get("out_collectives", 0) + 1
        state["out_exchanged_bytes"] = state.get("out_exchanged_bytes", 0) + out_bytes
        state["effective_comm_dtype"] = str(dtype).replace("torch.", "")
        state["exchange"] = exchange

    def forward_token(self, x_q, x_k, x_v, w_q=None, w_k=None, freqs=None, *, total: int, heads: int,
                      eps: float = 1e-6, scale: float | None = None, out_dtype: torch.dtype | None = None,
                      norm_rope: bool = True, state: dict | None = None,
                      rope_split_pairs: int | None = None) -> torch.Tensor:
        """Token mode (the reference's sequence_mode="token",
        powershard/wan_model.py:489-500): keys/values of every rank are
        all-gathered, queries stay local, so no output exchange is needed.

        Same inputs and output as ``forward``; rank r owns rows
        shard_bounds(total, r, W).  Steps: pre-pass into the local block
        [3, width, H, D]; all-gather of its k/v part into [W, 2, width, H, D]
        (the rows of gather_tokens, wan_model.py:336-340 / attention.py:40-54,
        padded to equal width); attention of the local queries against the W
        key segments, written straight to the [n, H, D] output.  With the
        peer exchange the pre-pass stores the k/v rows straight into every
        rank's gathered buffer instead (two 4-byte all-reduces order it).
        """
        device = x_q.device
        dtype = x_q.dtype
        head_dim = x_q.shape[-1] if x_q.dim() == 3 else x_q.shape[-1] // heads
        world, rank = self.world_rank()
        a, b = shard_bounds(total, rank, world)
        n = b - a
        if x_q.shape[0] != n:
            raise ValueError("token mode: local token count does not match shard_bounds")
        width = -(-total // world)
        out_dtype = out_dtype or dtype
        scale = head_dim ** -0.5 if scale is None else float(scale)
        k = self.kernels
        with torch.cuda.device(device) if device.type == "cuda" else contextlib.nullcontext():
            status = self._device_status(device)
            status.poll()
            stream = torch.cuda.current_stream(device).cuda_stream if device.type == "cuda" else 0
            if world > 1:
                geo = UlyssesGeometry(total=total, heads=heads, head_dim=head_dim, world=world, rank=rank)
                px = self._peer(geo, dtype, device, layout="token")
                if px is not None:
                    # k/v rows stored straight into every rank's gathered buffer.
                    qkey = ("token_q", device.index, stream, width, heads, head_dim, dtype)
                    if qkey not in self._buffers:
                        self._buffers[qkey] = torch.empty((width, heads, head_dim), dtype=dtype, device=device)
                    q_loc = self._buffers[qkey]
                    k.token_pack_to(x_q, x_k, x_v, w_q, w_k, freqs, q_loc, px.kv_dst, n, heads, head_dim, eps,
                                    norm_rope, **self._rope_kw(rope_split_pairs))
                    px.barrier()
                    out = torch.empty((n, heads, head_dim), dtype=out_dtype, device=device)
                    k.token_attention(q_loc, px.kv_all, out, n, total, scale, status, **self._ws(device))
                    px.barrier()
                    self._count_token(state, total, heads, head_dim, dtype, "peer")
                    return out
            key = ("token", device.index, stream, world, width, heads, head_dim, dtype)
            tb = self._buffers.get(key)
            if tb is None:
                tb = self._buffers[key] = dict(
                    qkv=torch.empty((3, width, heads, head_dim), dtype=dtype, device=device),
                    kv_all=torch.empty((world if world > 1 else 0, 2, width, heads, head_dim), dtype=dtype,
                                       device=device))
            k.token_pack(x_q, x_k, x_v, w_q, w_k, freqs, tb["qkv"], n, heads, head_dim, eps, norm_rope,
                         **self._rope_kw(rope_split_pairs))
            if world > 1:
                kv = tb["kv_all"]
                dist.all_gather_into_tensor(kv.view(world * 2 * width, heads, head_dim),
                                            tb["qkv"][1:].view(2 * width, heads, head_dim), group=self.group)
            else:
                kv = tb["qkv"][1:].unsqueeze(0)  # one segment: this rank's own rows
            out = torch.empty((n, heads, head_dim), dtype=out_dtype, device=device)
            k.token_attention(tb["qkv"], kv, out, n, total, scale, status, **self._ws(device))
        self._count_token(state, total, heads, head_dim, dtype, "nccl" if world > 1 else "local")
        return out

    def _count_token(self, state, total, heads, head_dim, dtype, exchange, batch=1):
        self.last_exchange = exchange
        self.count_token(state, total, heads, head_dim, dtype, exchange, batch)

    @staticmethod
    def count_token(state, total, heads, head_dim, dtype, exchange, batch=1):
        """Token-mode counters (wan_model.py:489-500): one K/V gather per block,
        the gathered [B, total, 2, H, D] bytes."""
        if state is None:
            return
        state["kv_collectives"] = state.get("kv_collectives", 0) + 1
        state["kv_gathered_bytes"] = (state.get("kv_gathered_bytes", 0)
                                      + 2 * batch * total * heads * head_dim * dtype.itemsize)
        state["effective_comm_dtype"] = str(dtype).replace("torch.", "")
        state["exchange"] = exchange

    def forward_joint(self, txt, img, w_q=None, w_k=None, txt_freqs=None, img_freqs=None, *, total_img: int,
                      heads: int, eps: float = 1e-6, scale: float | None = None,
                      out_dtype: torch.dtype | None = None, norm: int = ops.NORM_PER_HEAD,
                      state: dict | None = None, sizes=None, out=None):
        """Flux joint attention: text rows replicated on every rank, image rows Ulysses-split.

        txt = (q, k, v) [P, H*D] (or [P, H, D], any row/head strides)
        projections of the P text tokens (identical on every rank); img =
        (q, k, v) [n_img_local, H*D] of this rank's image tokens: the
        shard_bounds part of total_img, or part `rank` of `sizes` (the image
        Layout's balanced split).  With norm NORM_PER_HEAD, w_q/w_k [D] are
        the QK-norm weights and txt_freqs [P, D/2, 2, 2] / img_freqs
        [n_img_local, D/2, 2, 2] the rotation tables; with NORM_NONE the
        inputs are already normalised/rotated and only exchanged.  Keys and
        queries of every head are [text; all image tokens].  Only image rows
        cross the all-to-all; each rank attends text queries for its own
        heads and the text outputs are all-gathered over heads.  Returns
        (txt_out [P, H, D], img_out [n_img_local, H, D]) in out_dtype, written
        into `out` = (txt_out, img_out) when given (contiguous tensors).
        """
        device = img[0].device
        dtype = img[0].dtype
        head_dim = img[0].shape[-1] if img[0].dim() == 3 else img[0].shape[-1] // heads
        geo = self.geometry(total_img, heads, head_dim, sizes=sizes)
        if img[0].shape[0] != geo.n_local:
            raise ValueError("Ulysses local token/head geometry mismatch")
        plen = txt[0].shape[0]
        tgeo = UlyssesGeometry.replicated(plen, heads, head_dim, geo.world)
        out_dtype = out_dtype or dtype
        scale = head_dim ** -0.5 if scale is None else float(scale)
        k = self.kernels
        with torch.cuda.device(device) if device.type == "cuda" else contextlib.nullcontext():
            ws, status = self._workspace(geo, dtype, device)
            status.poll()
            stream = torch.cuda.current_stream(device).cuda_stream if device.type == "cuda" else 0
            tkey = ("txt", device.index, stream, plen, geo.world, geo.heads_per_rank, head_dim, dtype)
            if tkey not in self._buffers:  # text rows: packed q/k/v and this rank's heads' outputs (wire dtype)
                self._buffers[tkey] = dict(
                    send=torch.empty(tgeo.send_shape(), dtype=dtype, device=device),
                    out=torch.empty((plen, geo.heads_per_rank, head_dim), dtype=dtype, device=device),
                    gathered=torch.empty((geo.world * plen, geo.heads_per_rank, head_dim), dtype=dtype,
                                         device=device))  # concatenated along dim 0 (any backend)
            tb = self._buffers[tkey]
            if out is not None:
                txt_out, img_out = out
                for t, rows in ((txt_out, plen), (img_out, geo.n_local)):
                    if tuple(t.shape) != (rows, heads, head_dim) or not t.is_contiguous() or t.dtype != out_dtype:
                        raise ValueError(f"forward_joint: out tensors must be contiguous [{rows}, {heads}, "
                                         f"{head_dim}] {out_dtype}")
            else:
                img_out = torch.empty((geo.n_local, heads, head_dim), dtype=out_dtype, device=device)
                txt_out = torch.empty((plen, heads, head_dim), dtype=out_dtype, device=device)
            px = self._peer(geo, dtype, device, text_rows=plen)
            if px is not None:
                # Image rows cross by peer stores, the text outputs of this
                # rank's heads are copied into every rank's text buffer.
                if plen:
                    k.prepass(*txt, w_q, w_k, txt_freqs, tb["send"], tgeo, eps, norm)
                k.prepass_to(*img, w_q, w_k, img_freqs, px.dst_blocks, geo, dtype, eps, norm)
                px.barrier()
                k.ulysses_joint_attention_to(px.recv, tb["send"][geo.rank], px.out_blocks, px.out_row_stride,
                                             tb["out"], dtype, geo, scale, status, **self._ws(device))
                if plen:
                    k.broadcast(px.text_dst, tb["out"])
                px.barrier()
                k.unpack_staged(px.staging, img_out, geo)
                if plen:
                    k.unpack(px.text.view(tgeo.out_shape()), txt_out, tgeo)
                self._count_joint(state, geo, dtype, "peer")
                return txt_out, img_out
            if plen:
                k.prepass(*txt, w_q, w_k, txt_freqs, tb["send"], tgeo, eps, norm)
            k.prepass(*img, w_q, w_k, img_freqs, ws["send"], geo, eps, norm)
            self._exchange(ws["recv"], ws["send"], geo)
            prefix = tb["send"][geo.rank]
            if geo.world == 1:
                k.ulysses_joint_attention(ws["recv"], prefix, img_out.view(geo.out_shape()), txt_out, geo, scale,
                                          status, **self._ws(device))
            else:
                k.ulysses_joint_attention(ws["recv"], prefix, ws["out_send"], tb["out"], geo, scale, status,
                                          **self._ws(device))
                self._exchange(ws["out_recv"], ws["out_send"], geo)
                k.unpack(ws["out_recv"], img_out, geo)
                if plen:
                    dist.all_gather_into_tensor(tb["gathered"], tb["out"], group=self.group)
                    k.unpack(tb["gathered"].view(tgeo.out_shape()), txt_out, tgeo)
        self._count_joint(state, geo, dtype, "nccl" if geo.world > 1 else "local")
        return txt_out, img_out

    @staticmethod
    def _count_joint(state, geo, dtype, exchange):
        if state is None:
            return
        qkv_bytes, out_bytes = geo.exchanged_bytes(dtype.itemsize)
        state["padded_heads"] = geo.padded_heads
        state["kv_collectives"] = state.get("kv_collectives", 0) + 1
        state["kv_gathered_bytes"] = state.get("kv_gathered_bytes", 0) + qkv_bytes
        state["out_collectives"] = state.get("out_collectives", 0) + 2
        state["out_exchanged_bytes"] = state.get("out_exchanged_bytes", 0) + out_bytes
        state["exchange"] = exchange

    def check(self):
        """Synchronize and raise if any attention launch aborted on the device."""
        for status in self._status.values():
            status.check()
