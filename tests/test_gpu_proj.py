"""Projection GEMMs on the CUDA path (needs a B200), through the C ABI.

* ps_b200_out_proj: y = A W^T + b against a torch fp32 matmul of the same
  bf16 operands, with A as plain rows, as the peer exchange's staging rows
  (row stride above the width) and as the NCCL receive buffer's per-source
  blocks; fp32 output within fp32-accumulation error, bf16 output within one
  bf16 rounding.
* ps_b200_qkv_proj: the send blocks against a torch restatement of the
  reference's attention_qkv (powershard/wan_model.py:421-430) on the fp32
  projection - RMSNorm over the full width rounded to the wire type, then
  RoPE, as the pre-pass kernel computes it - within 2 bf16 ulps per element
  (accumulation and summation order), with padding rows and head slots zero.
"""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def _ref_matmul(a, w, b):
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        y = a.float() @ w.float().t()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    return y if b is None else y + b.float()


@pytest.mark.parametrize("n,fin,fout,dtype", [(1, 64, 256, torch.bfloat16), (300, 512, 512, torch.bfloat16),
                                              (1000, 1536, 1536, torch.bfloat16), (4095, 5120, 5120, torch.bfloat16),
                                              (700, 768, 512, torch.float16), (257, 512, 256, torch.float16)])
def test_out_projection_rows(cuda_lib, n, fin, fout, dtype):
    """fp32 output against torch's fp32 matmul; the 16-bit output is exactly
    the fp32 output rounded once (same accumulation, one rounding)."""
    from powershard_b200 import ops
    g = torch.Generator(device=DEV).manual_seed(n + fin)
    a = torch.randn(n, fin, device=DEV, generator=g).to(dtype)
    w = (torch.randn(fout, fin, device=DEV, generator=g) * 0.02).to(dtype)
    b = torch.randn(fout, device=DEV, generator=g) * 0.1
    out32 = torch.empty(n, fout, device=DEV, dtype=torch.float32)
    out16 = torch.empty(n, fout, device=DEV, dtype=dtype)
    status = ops.DeviceStatus(DEV)
    ops.out_projection(a, w, b, out32, n, fin, a.stride(0), status=status)
    ops.out_projection(a, w, b, out16, n, fin, a.stride(0), status=status)
    status.check()
    ref = _ref_matmul(a, w, b)
    assert float((out32 - ref).abs().max()) <= 1e-3 * max(1.0, float(ref.abs().max()))
    assert torch.equal(out16, out32.to(dtype))


def test_out_projection_from_exchange_buffers(cuda_lib):
    """A read in place from the peer staging layout [width][W*h][D] (first H*D
    columns) and from the NCCL receive layout [W][width][h][D]."""
    from powershard_b200 import ops
    world, width, heads, hpr, d = 3, 700, 5, 2, 128
    n = width - 11
    g = torch.Generator(device=DEV).manual_seed(3)
    rows = torch.randn(n, heads * d, device=DEV, generator=g).bfloat16()
    w = (torch.randn(512, heads * d, device=DEV, generator=g) * 0.02).bfloat16()
    ref = _ref_matmul(rows, w, None)
    status = ops.DeviceStatus(DEV)
    # staging rows: [width][W*h][D], heads in order, padded slots after them
    staging = torch.zeros(width, world * hpr, d, device=DEV, dtype=torch.bfloat16)
    staging[:n, :heads] = rows.view(n, heads, d)
    out = torch.empty(n, 512, device=DEV)
    ops.out_projection(staging, w, None, out, n, heads * d, world * hpr * d, status=status)
    status.check()
    torch.testing.assert_close(out, ref, atol=2e-3, rtol=2e-3)
    # NCCL receive layout: block s holds heads [s*h, (s+1)*h) of every row
    recv = torch.zeros(world, width, hpr, d, device=DEV, dtype=torch.bfloat16)
    padded = torch.zeros(n, world * hpr, d, device=DEV, dtype=torch.bfloat16)
    padded[:, :heads] = rows.view(n, heads, d)
    recv[:, :n] = padded.view(n, world, hpr, d).transpose(0, 1)
    out2 = torch.empty(n, 512, device=DEV)
    ops.out_projection(recv, w, None, out2, n, heads * d, hpr * d, block_stride=width * hpr * d, block_cols=hpr * d,
                       status=status)
    status.check()
    torch.testing.assert_close(out2, ref, atol=2e-3, rtol=2e-3)


def _qkv_reference(x, ws, bs, nq, nk, table, heads, eps=1e-6):
    """attention_qkv on the fp32 projections: RMSNorm rounded to the wire
    type, RoPE in fp32, cast to the wire; v is the projection rounded once."""
    wire = x.dtype
    outs = []
    for i, (w, b) in enumerate(zip(ws, bs)):
        y = _ref_matmul(x, w, b)
        if i < 2:
            nw = (nq, nk)[i].float()
            y = (y * torch.rsqrt(y.square().mean(-1, keepdim=True) + eps) * nw).to(wire).float()
            y = y.view(y.shape[0], heads, -1, 1, 2)
            rot = table[:, None]
            y = (rot[..., 0] * y[..., 0] + rot[..., 1] * y[..., 1]).reshape(y.shape[0], heads, -1)
        else:
            y = y.view(y.shape[0], heads, -1)
        outs.append(y.to(wire))
    return outs


@pytest.mark.parametrize("total,heads,world,fin,dtype", [(300, 4, 1, 512, torch.bfloat16),
                                                         (1000, 12, 2, 1536, torch.bfloat16),
                                                         (41, 6, 4, 256, torch.bfloat16),
                                                         (4095, 40, 1, 5120, torch.bfloat16),
                                                         (1500, 40, 8, 5120, torch.bfloat16),
                                                         (700, 8, 2, 1024, torch.float16)])
def test_qkv_projection_matches_attention_qkv(cuda_lib, total, heads, world, fin, dtype):
    from powershard_b200 import ops
    from powershard_b200.partition import UlyssesGeometry
    from powershard_b200.rope import rope_table_3d
    d = 128
    g = torch.Generator(device=DEV).manual_seed(total + heads)
    x_all = torch.randn(total, fin, device=DEV, generator=g).to(dtype)
    ws = [(torch.randn(heads * d, fin, device=DEV, generator=g) * 0.02).to(dtype) for _ in range(3)]
    bs = [torch.randn(heads * d, device=DEV, generator=g) * 0.05 for _ in range(3)]
    nq = torch.rand(heads * d, device=DEV, generator=g) + 0.5
    nk = torch.rand(heads * d, device=DEV, generator=g) + 0.5
    side = max(1, round(total ** (1 / 3)))
    table = rope_table_3d((math.ceil(total / side ** 2), side, side), d, device=DEV)[:total].contiguous()
    refs = _qkv_reference(x_all, ws, bs, nq, nk, table, heads)
    status = ops.DeviceStatus(DEV)
    for rank in range(world):
        geo = UlyssesGeometry(total=total, heads=heads, head_dim=d, world=world, rank=rank)
        a, b = geo.bounds
        send = torch.full(geo.send_shape(), float("nan"), device=DEV, dtype=dtype)
        wsp = ops.projection_workspace(geo.n_local, heads, d, DEV)
        ops.qkv_projection(x_all[a:b], *ws, *bs, nq, nk, table[a:b], ops.send_blocks(send), geo, 1e-6, wsp,
                           status)
        status.check()
        assert bool(torch.isfinite(send).all()), "padding rows / head slots must be written as zeros"
        h = geo.heads_per_rank
        flat = send.permute(1, 2, 0, 3, 4).reshape(3, geo.width, world * h, d)
        assert not flat[:, b - a:].any() and not flat[:, :, heads:].any()
        ulp = 2.0 ** -7 if dtype == torch.bfloat16 else 2.0 ** -10
        for kind in range(3):
            got = flat[kind, :b - a, :heads].float()
            want = refs[kind][a:b].float()
            diff = (got - want).abs()
            assert bool((diff <= ulp * (2 * want.abs() + 4)).all()), f"kind {kind}: max {float(diff.max()):.3e}"
            assert float((got == want).float().mean()) >= 0.9


def test_qkv_projection_peer_style_destinations(cuda_lib):
    """Destinations given as separate buffers (as the peer exchange gives the
    other ranks' receive blocks) receive the same bytes as one send buffer."""
    from powershard_b200 import ops
    from powershard_b200.partition import UlyssesGeometry
    from powershard_b200.rope import rope_table_3d
    total, heads, world, fin, d = 900, 8, 4, 1024, 128
    g = torch.Generator(device=DEV).manual_seed(5)
    geo = UlyssesGeometry(total=total, heads=heads, head_dim=d, world=world, rank=2)
    a, b = geo.bounds
    x = torch.randn(b - a, fin, device=DEV, generator=g).bfloat16()
    ws = [(torch.randn(heads * d, fin, device=DEV, generator=g) * 0.02).bfloat16() for _ in range(3)]
    nw = torch.ones(heads * d, device=DEV)
    table = rope_table_3d((9, 10, 10), d, device=DEV)[a:b].contiguous()
    wsp = ops.projection_workspace(geo.n_local, heads, d, DEV)
    send = torch.empty(geo.send_shape(), device=DEV, dtype=torch.bfloat16)
    ops.qkv_projection(x, *ws, None, None, None, nw, nw, table, ops.send_blocks(send), geo, 1e-6, wsp)
    blocks = [torch.empty(geo.send_shape()[1:], device=DEV, dtype=torch.bfloat16) for _ in range(world)]
    ops.qkv_projection(x, *ws, None, None, None, nw, nw, table, [t.data_ptr() for t in blocks], geo, 1e-6, wsp)
    torch.cuda.synchronize()
    for dst in range(world):
        assert torch.equal(blocks[dst], send[dst])
