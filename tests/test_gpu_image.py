"""Image-model (Flux) sequence parallelism on the CUDA path (needs a B200).

The image Layout splits the image segment evenly (the first n % W ranks one
row longer), so a source segment of the receive buffer can be short in the
middle of the sequence, not only at its tail.  These tests drive the
per-segment row table through the C ABI (plain and joint attention), and the
``SequenceAttention`` override end to end: alone at W = 1 and with W ranks
emulated on one GPU by threads whose collectives are in-process copies
(every kernel still runs; ranks never wait on each other inside a kernel).
Tolerance: max |err| <= 2e-2 and mean |err| / mean |ref| <= 5e-3 against
the fp32 oracle.
"""
import pytest
import torch
from emulated_dist import emulated_group

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
MAX_ABS, MEAN_REL = 2e-2, 5e-3
PAD = 64.0  # finite garbage in padding rows: a key that leaks in dominates its row's softmax


def assert_attention_close(got, ref):
    got, ref = got.float().cpu(), ref.float().cpu()
    assert got.shape == ref.shape
    assert torch.isfinite(got).all()
    err = (got - ref).abs()
    rel = float(err.mean() / ref.abs().mean().clamp_min(1e-12))
    assert float(err.max()) <= MAX_ABS and rel <= MEAN_REL, f"max_abs={float(err.max()):.3e} mean_rel={rel:.3e}"


def balanced_recv(geo, q, k, v, dtype=torch.bfloat16):
    """Receive buffer [W,3,width,h,D] of geo.rank's heads for full q/k/v
    [total, H, D] split by geo.sizes; padding rows hold PAD."""
    from powershard_b200.partition import UlyssesGeometry
    h, world = geo.heads_per_rank, geo.world
    recv = torch.full(geo.send_shape(), PAD, dtype=dtype)
    lo = geo.rank * h
    hv = geo.heads_valid
    for s in range(world):
        a, b = UlyssesGeometry(geo.total, geo.heads, 128, world, s, geo.sizes).bounds
        for kind, t in enumerate((q, k, v)):
            recv[s, kind, :b - a, :hv] = t[a:b, lo:lo + hv].to(dtype)
            recv[s, kind, :b - a, hv:] = 0
    return recv


@pytest.mark.parametrize("image,heads,world", [(1001, 6, 5), (1001, 8, 4), (4097, 3, 3), (260, 2, 7)])
def test_attention_with_balanced_segments(cuda_lib, oracle, image, heads, world):
    from powershard_b200 import ops
    from powershard_b200.partition import UlyssesGeometry, split_sizes
    sizes = split_sizes(image, world)
    g = torch.Generator().manual_seed(5)
    q, k, v = (torch.randn(image, heads, 128, generator=g) for _ in range(3))
    ref = oracle.sdpa_fp32(*(t.bfloat16().float()[None] for t in (q, k, v)))[0]
    for rank in range(world):
        geo = UlyssesGeometry(image, heads, 128, world, rank, tuple(sizes))
        if not geo.heads_valid:
            continue
        recv = balanced_recv(geo, q, k, v).to(DEV)
        out = torch.full(geo.out_shape(), -7.0, dtype=torch.bfloat16, device=DEV)
        status = ops.DeviceStatus(DEV)
        ops.ulysses_attention(recv, out, geo, 128 ** -0.5, status)
        status.check()
        out = out.cpu()
        row, lo = 0, rank * geo.heads_per_rank
        for s, n in enumerate(sizes):
            assert_attention_close(out[s, :n, :geo.heads_valid], ref[row:row + n, lo:lo + geo.heads_valid])
            assert (out[s, n:] == -7.0).all(), "rows past a segment's valid count must stay untouched"
            row += n


@pytest.mark.parametrize("prefix,image,heads,world", [(512, 4097, 3, 3), (77, 1001, 6, 5), (5, 260, 2, 7)])
def test_joint_attention_with_balanced_segments(cuda_lib, oracle, prefix, image, heads, world):
    from powershard_b200 import ops
    from powershard_b200.partition import UlyssesGeometry, split_sizes
    sizes = split_sizes(image, world)
    g = torch.Generator().manual_seed(6)
    full = [torch.randn(prefix + image, heads, 128, generator=g) for _ in range(3)]
    ref = oracle.sdpa_fp32(*(t.bfloat16().float()[None] for t in full))[0]
    for rank in range(world):
        geo = UlyssesGeometry(image, heads, 128, world, rank, tuple(sizes))
        if not geo.heads_valid:
            continue
        h, hv, lo = geo.heads_per_rank, geo.heads_valid, rank * geo.heads_per_rank
        recv = balanced_recv(geo, *(t[prefix:] for t in full)).to(DEV)
        pre = torch.zeros(3, prefix, h, 128, dtype=torch.bfloat16)
        for kind in range(3):
            pre[kind, :, :hv] = full[kind][:prefix, lo:lo + hv].bfloat16()
        out = torch.full(geo.out_shape(), -7.0, dtype=torch.bfloat16, device=DEV)
        pout = torch.zeros(prefix, h, 128, dtype=torch.bfloat16, device=DEV)
        status = ops.DeviceStatus(DEV)
        ops.ulysses_joint_attention(recv, pre.to(DEV), out, pout, geo, 128 ** -0.5, status)
        status.check()
        assert_attention_close(pout.cpu()[:, :hv], ref[:prefix, lo:lo + hv])
        out = out.cpu()
        row = prefix
        for s, n in enumerate(sizes):
            assert_attention_close(out[s, :n, :hv], ref[row:row + n, lo:lo + hv])
            assert (out[s, n:] == -7.0).all()
            row += n


# ------------------------------------------------ override, ranks emulated
def _local(oracle, t, segments, world, rank, heads, skip):
    """Rank's local rows of a full [B, L, H, D] tensor in the block layout."""
    rows = [i for s, e in oracle.image_local_ranges(segments, world, rank) for i in range(s, e)]
    x = t[:, rows]
    if skip:
        return x.transpose(1, 2).contiguous()     # [B, H, n, D]
    return x.reshape(x.shape[0], len(rows), heads * 128).contiguous()


@pytest.mark.parametrize("world,prefix,image,heads,batch,skip", [
    (1, 512, 4096, 24, 1, True),      # configs[4] shape, one rank
    (2, 512, 4096, 24, 1, True),      # configs[4] at W = 2
    (3, 512, 4097, 24, 1, True),      # balanced split [1366, 1366, 1365]
    (5, 77, 1001, 6, 2, False),       # short middle segments, batch 2, [B, L, H*D] inputs
    (4, 0, 1001, 6, 1, True),         # no text rows, padded heads
])
def test_sequence_attention_override(cuda_lib, oracle, world, prefix, image, heads, batch, skip):
    from powershard_b200.image import SequenceAttention
    from powershard_b200.partition import ImageLayout
    from powershard_b200.ulysses import UlyssesAttention
    segments = [(prefix, False), (image, True)]
    g = torch.Generator().manual_seed(12)
    full = [torch.randn(batch, prefix + image, heads, 128, generator=g).bfloat16() for _ in range(3)]
    expected = oracle.image_sequence_attention(*(t.float() for t in full), segments, world)

    def rank_fn(rank):
        lay = ImageLayout(segments, world, rank)
        stats = {}
        override = SequenceAttention(lay, stats, UlyssesAttention())
        local = [_local(oracle, t, segments, world, rank, heads, skip).to(DEV) for t in full]
        out = override(None, *local, heads, skip_reshape=skip)
        override.engine.check()
        assert stats["attention_calls"] == 1
        return out.cpu()

    if world == 1:
        outs = [rank_fn(0)]
    else:
        with emulated_group(world) as run:
            outs = run(rank_fn)
    for rank, out in enumerate(outs):
        ref = expected[rank]
        assert out.shape == (batch, ref.shape[1], heads * 128) and out.dtype == torch.bfloat16
        assert_attention_close(out, ref.reshape(out.shape))


def test_sequence_attention_override_output_layout_and_fallback(cuda_lib, oracle):
    from powershard_b200.contract import UnsupportedAttention
    from powershard_b200.image import SequenceAttention
    from powershard_b200.partition import ImageLayout
    segments = [(40, False), (300, True)]
    lay = ImageLayout(segments, 1, 0)
    g = torch.Generator().manual_seed(2)
    q, k, v = (torch.randn(1, 3, 340, 128, generator=g).bfloat16().to(DEV) for _ in range(3))
    override = SequenceAttention(lay, {})
    flat = override(None, q, k, v, 3, skip_reshape=True)
    bhld = override(None, q, k, v, 3, skip_reshape=True, skip_output_reshape=True)
    assert bhld.shape == (1, 3, 340, 128)
    assert torch.equal(bhld.transpose(1, 2).reshape(1, 340, 384), flat)
    mask = torch.zeros(340, 340, device=DEV)
    with pytest.raises(UnsupportedAttention):
        override(None, q, k, v, 3, mask, skip_reshape=True)
    seen = []
    fallback = SequenceAttention(lay, {}, fallback=lambda func, *a, **kw: seen.append(kw) or "fallback")
    assert fallback(None, q, k, v, 3, mask=mask, skip_reshape=True) == "fallback" and seen
    with pytest.raises(UnsupportedAttention):  # keys appended inside the attention
        override(None, q, torch.cat([k, k[:, :, :4]], 2), torch.cat([v, v[:, :, :4]], 2), 3, skip_reshape=True)
    with pytest.raises(ValueError):  # wrong local length
        override(None, q[:, :, :300], k, v, 3, skip_reshape=True)
