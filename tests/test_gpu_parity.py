"""CUDA path vs the CPU oracle, through the C ABI (needs a B200).

Tolerances:
* pre-pass (RMSNorm + RoPE + pack): each element within 2 bf16/fp16 ulps of
  the oracle (the only difference is the summation order of mean(x^2)),
  >= 99% bit-identical, padding exactly zero;
* attention / whole block: the north-star bound against the fp32 oracle,
  max |err| <= 2e-2 and mean |err| / mean |ref| <= 5e-3.
"""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
MAX_ABS, MEAN_REL = 2e-2, 5e-3


def assert_attention_close(got, ref, max_abs=MAX_ABS, mean_rel=MEAN_REL):
    got, ref = got.float().cpu(), ref.float().cpu()
    assert got.shape == ref.shape
    assert torch.isfinite(got).all()
    err = (got - ref).abs()
    rel = float(err.mean() / ref.abs().mean().clamp_min(1e-12))
    assert float(err.max()) <= max_abs and rel <= mean_rel, f"max_abs={float(err.max()):.3e} mean_rel={rel:.3e}"


def geometry(total, heads, world, rank):
    from powershard_b200.partition import UlyssesGeometry
    return UlyssesGeometry(total=total, heads=heads, head_dim=128, world=world, rank=rank)


def rank_inputs(oracle, total, heads, seed, dtype, scale=1.5):
    g = torch.Generator().manual_seed(seed)
    x = [(torch.randn(1, total, heads * 128, generator=g) * scale).to(dtype) for _ in range(3)]
    wq = torch.rand(heads * 128, generator=g) + 0.5
    wk = torch.rand(heads * 128, generator=g) + 0.5
    side = max(1, round(total ** (1 / 3)))
    grid = (math.ceil(total / (side * side)), side, side)
    freqs = oracle.rope_table_3d(grid, 128)[:, :total]
    return x, wq, wk, freqs


# ------------------------------------------------------------------- pre-pass
@pytest.mark.parametrize("total,heads,world", [(300, 4, 1), (37, 5, 2), (41, 7, 3), (9, 3, 4), (130, 40, 8)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("wdtype", ["fp32", "same"])
def test_prepass_matches_oracle(cuda_lib, oracle, total, heads, world, dtype, wdtype):
    from powershard_b200 import ops
    x, wq, wk, freqs = rank_inputs(oracle, total, heads, 3, dtype)
    if wdtype == "same":
        wq, wk = wq.to(dtype), wk.to(dtype)
    ulp = 2.0 ** -7 if dtype == torch.bfloat16 else 2.0 ** -10
    for rank in range(world):
        geo = geometry(total, heads, world, rank)
        a, b = geo.bounds
        send = torch.full(geo.send_shape(), float("nan"), dtype=dtype, device=DEV)
        ops.prepass(*(t[0, a:b].to(DEV) for t in x), wq.to(DEV), wk.to(DEV), freqs[0, a:b, 0].to(DEV), send, geo)
        q, k, v = oracle.attention_qkv(x[0][:, a:b], x[1][:, a:b], x[2][:, a:b], wq, wk, freqs[:, a:b], heads)
        expected = oracle.pack_qkv(q[0].to(dtype), k[0].to(dtype), v[0].to(dtype), total, rank, world)
        got = send.cpu()
        assert torch.isfinite(got).all(), "padding must be written (zeros)"
        diff = (got.float() - expected.float()).abs()
        # One ulp of the normalised pair (|y| <= ~4) plus the final rounding.
        bound = ulp * (2 * expected.float().abs() + 4)
        assert bool((diff <= bound).all()), f"rank {rank}: max diff {float(diff.max()):.3e}"
        assert float((got == expected).float().mean()) >= 0.99
        assert torch.equal(got[:, 2], expected[:, 2]), "v is a copy"
        # zero padding: heads >= H and rows >= n_local
        h = geo.heads_per_rank
        flat = got.permute(1, 2, 0, 3, 4).reshape(3, geo.width, world * h, 128)
        assert not flat[:, :, heads:].any()
        assert not flat[:, b - a:].any()


def test_prepass_pack_only_is_exact(cuda_lib, oracle):
    from powershard_b200 import ops
    total, heads, world = 50, 6, 4
    g = torch.Generator().manual_seed(5)
    q, k, v = (torch.randn(total, heads, 128, generator=g).to(torch.bfloat16) for _ in range(3))
    for rank in range(world):
        geo = geometry(total, heads, world, rank)
        a, b = geo.bounds
        send = torch.empty(geo.send_shape(), dtype=torch.bfloat16, device=DEV)
        ops.prepass(*(t[a:b].reshape(b - a, -1).to(DEV) for t in (q, k, v)), None, None, None, send, geo,
                    norm_rope=False)
        expected = oracle.pack_qkv(q[a:b], k[a:b], v[a:b], total, rank, world)
        assert torch.equal(send.cpu(), expected)


# ------------------------------------------------------------------ attention
def oracle_recv(oracle, total, heads, world, seed, dtype=torch.bfloat16):
    """Per-rank receive buffers built by the oracle (pack + all-to-all)."""
    g = torch.Generator().manual_seed(seed)
    q, k, v = (torch.randn(total, heads, 128, generator=g) for _ in range(3))
    sends = []
    for r in range(world):
        a, b = oracle.shard_bounds(total, r, world)
        sends.append(oracle.pack_qkv(q[a:b].to(dtype), k[a:b].to(dtype), v[a:b].to(dtype), total, r, world))
    return oracle.exchange(sends)


@pytest.mark.parametrize("total,heads,world", [(1, 1, 1), (127, 2, 1), (129, 2, 1), (300, 3, 1), (1000, 2, 1),
                                               (37, 5, 2), (9, 3, 4), (257, 3, 3), (1100, 4, 2), (2 * 7 + 1, 7, 7)])
def test_ulysses_attention_matches_oracle(cuda_lib, oracle, total, heads, world):
    from powershard_b200 import ops
    recvs = oracle_recv(oracle, total, heads, world, 11)
    for rank in range(world):
        geo = geometry(total, heads, world, rank)
        status = ops.DeviceStatus(DEV)
        out = torch.zeros(geo.out_shape(), dtype=torch.bfloat16, device=DEV)
        ops.ulysses_attention(recvs[rank].to(DEV), out, geo, 128 ** -0.5, status)
        status.check()
        q, k, v = oracle.unpack_qkv(recvs[rank], total)
        ref = oracle.sdpa_fp32(q[None], k[None], v[None])[0]          # [total, h, D]
        hv = geo.heads_valid
        got = out.cpu().reshape(world * geo.width, geo.heads_per_rank, 128)[:total, :hv]
        if hv:
            assert_attention_close(got, ref[:, :hv])


def test_ulysses_attention_fp32_output(cuda_lib, oracle):
    from powershard_b200 import ops
    total, heads = 500, 2
    recv = oracle_recv(oracle, total, heads, 1, 4)[0]
    geo = geometry(total, heads, 1, 0)
    out = torch.zeros(geo.out_shape(), dtype=torch.float32, device=DEV)
    ops.ulysses_attention(recv.to(DEV), out, geo, 0.07, None)
    q, k, v = oracle.unpack_qkv(recv, total)
    assert_attention_close(out.cpu()[0], oracle.sdpa_fp32(q[None], k[None], v[None], 0.07)[0])


@pytest.mark.parametrize("slope", [0.5, 4.0, 12.0, -6.0])
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
def test_running_max_rescale_paths(cuda_lib, oracle, slope, out_dtype):
    """Scores that grow (or shrink) steadily along the keys: the row max rises
    by `slope` log2 units per 32 keys, so the softmax raises its running max
    inside key tiles at every chunk position - before the first half of P is
    released, and after it (where O is scaled once that half's PV has run)."""
    from powershard_b200 import ops
    total, heads = 1000, 2
    geo = geometry(total, heads, 1, 0)
    g = torch.Generator().manual_seed(31)
    u = torch.randn(128, generator=g)
    u = u / u.norm()
    # q . k / sqrt(D) * log2(e) = slope / 32 per key step along the direction u
    step = slope / 32 / math.log2(math.e) * math.sqrt(128)
    q = (u * 4.0).expand(total, heads, 128).clone() + 0.05 * torch.randn(total, heads, 128, generator=g)
    pos = torch.arange(total, dtype=torch.float32)[:, None, None]
    k = u * (pos * step / 4.0) + 0.05 * torch.randn(total, heads, 128, generator=g)
    v = torch.randn(total, heads, 128, generator=g)
    recv = torch.stack([q, k, v])[None].bfloat16()           # [1, 3, total, h, D]
    out = torch.zeros(geo.out_shape(), dtype=out_dtype, device=DEV)
    status = ops.DeviceStatus(DEV)
    ops.ulysses_attention(recv.to(DEV), out, geo, 128 ** -0.5, status, workspace=ops.attention_workspace(DEV))
    status.check()
    qb, kb, vb = (t.float() for t in recv[0])
    ref = oracle.sdpa_fp32(qb[None], kb[None], vb[None])[0]
    assert_attention_close(out.cpu()[0], ref)


def _split_of(units: int, key_tiles: int, sms: int) -> int:
    """The split the library picks for the last wave (mirror of its plan)."""
    rem = units % sms
    if rem == 0:
        return 1
    split = min(sms // rem, 8, key_tiles // 2)
    return split if split >= 2 else 1


@pytest.mark.parametrize("total,heads,world,out_dtype", [
    (1000, 2, 1, torch.bfloat16),    # 8 units: split 4
    (4099, 3, 1, torch.bfloat16),    # 51 units: split 2
    (1000, 2, 1, torch.float32),     # fp32 output through the combine kernel
    (1001, 6, 4, torch.bfloat16),    # 4 source segments, 2 real heads per rank
    (130, 1, 1, torch.bfloat16),     # 2 key tiles: too few to split
])
def test_split_last_wave_matches_oracle(cuda_lib, oracle, total, heads, world, out_dtype):
    """With a workspace, the last partial wave's units run as several CTAs
    over parts of the key range and a combine kernel merges them by
    log-sum-exp: same bound against the oracle, and close to the unsplit
    launch."""
    from powershard_b200 import _lib, ops
    lib = _lib.load()
    recvs = oracle_recv(oracle, total, heads, world, 21)
    sms = torch.cuda.get_device_properties(DEV).multi_processor_count
    for rank in range(world):
        geo = geometry(total, heads, world, rank)
        if not geo.heads_valid:
            continue
        q_tiles = world * -(-geo.width // 128)
        key_tiles = sum(-(-v // 128) for v in geo.seg_valid())
        units = -(-q_tiles // 2) * geo.heads_valid
        recv = recvs[rank].to(DEV)
        outs = []
        for ws in (None, ops.attention_workspace(DEV)):
            out = torch.zeros(geo.out_shape(), dtype=out_dtype, device=DEV)
            status = ops.DeviceStatus(DEV)
            before = lib.ps_b200_kernel_launches()
            ops.ulysses_attention(recv, out, geo, 128 ** -0.5, status, workspace=ws)
            status.check()
            launched = lib.ps_b200_kernel_launches() - before
            expect_split = ws is not None and _split_of(units, key_tiles, sms) > 1
            assert launched == (2 if expect_split else 1)
            outs.append(out.float().cpu())
        q, k, v = oracle.unpack_qkv(recvs[rank], total)
        ref = oracle.sdpa_fp32(q[None], k[None], v[None])[0]
        hv = geo.heads_valid
        for out in outs:
            got = out.reshape(world * geo.width, geo.heads_per_rank, 128)[:total, :hv]
            assert_attention_close(got, ref[:, :hv])
        # Each part rounds its probabilities to bf16 against its own running
        # max, so split and unsplit differ at the level of that rounding.
        diff = (outs[0] - outs[1]).abs()
        assert float(diff.mean() / outs[0].abs().mean()) <= 2e-3 and float(diff.max()) <= 1e-2


def test_split_joint_prefix_matches_oracle(cuda_lib, oracle):
    """Split last wave with a text prefix range (Flux joint attention)."""
    from powershard_b200 import ops
    from powershard_b200.partition import UlyssesGeometry
    prefix, image, heads = 77, 1001, 2
    g = torch.Generator().manual_seed(9)
    full = [torch.randn(prefix + image, heads, 128, generator=g).bfloat16() for _ in range(3)]
    geo = UlyssesGeometry(image, heads, 128, 1, 0)
    recv = torch.stack([t[prefix:] for t in full])[None].contiguous().to(DEV)      # [1, 3, image, h, D]
    pre = torch.stack([t[:prefix] for t in full]).contiguous().to(DEV)             # [3, P, h, D]
    ref = oracle.sdpa_fp32(*(t.float()[None] for t in full))[0]
    for ws in (None, ops.attention_workspace(DEV)):
        out = torch.zeros(geo.out_shape(), dtype=torch.bfloat16, device=DEV)
        pout = torch.zeros(prefix, heads, 128, dtype=torch.bfloat16, device=DEV)
        status = ops.DeviceStatus(DEV)
        ops.ulysses_joint_attention(recv, pre, out, pout, geo, 128 ** -0.5, status, workspace=ws)
        status.check()
        assert_attention_close(pout, ref[:prefix])
        assert_attention_close(out[0], ref[prefix:])


@pytest.mark.parametrize("b,lq,lk,hq,hk,dtype,scale", [
    (2, 5, 7, 4, 4, torch.float16, .13), (2, 5, 7, 4, 4, torch.bfloat16, .37), (1, 1, 1, 1, 1, torch.bfloat16, None),
    (1, 300, 300, 3, 3, torch.bfloat16, None), (2, 200, 4099, 4, 2, torch.bfloat16, .05),
    (1, 513, 129, 8, 1, torch.float16, None), (3, 256, 256, 2, 2, torch.float16, 1.3)])
def test_provider_matches_oracle(cuda_lib, oracle, b, lq, lk, hq, hk, dtype, scale):
    from powershard_b200.contract import AttentionOptions
    from powershard_b200.provider import B200Provider
    g = torch.Generator().manual_seed(lq * 31 + lk)
    q = torch.randn(b, lq, hq, 128, generator=g).to(dtype)
    k = torch.randn(b, lk, hk, 128, generator=g).to(dtype)
    v = torch.randn(b, lk, hk, 128, generator=g).to(dtype)
    out = B200Provider()(q.to(DEV), k.to(DEV), v.to(DEV), AttentionOptions(softmax_scale=scale))
    assert out.shape == (b, lq, hq, 128) and out.dtype == dtype and out.device == DEV
    rep = hq // hk
    ref = oracle.sdpa_fp32(q, k.repeat_interleave(rep, 2), v.repeat_interleave(rep, 2), scale)
    assert_attention_close(out, ref)


def test_provider_noncontiguous_and_probe_geometry(cuda_lib, oracle):
    from powershard_b200.contract import AttentionOptions
    from powershard_b200.provider import B200Provider
    g = torch.Generator().manual_seed(1729)
    q = torch.randn(2, 5, 4, 256, generator=g).half()[..., ::2]
    k = torch.randn(2, 7, 4, 128, generator=g).half()
    v = torch.randn(2, 7, 4, 128, generator=g).half()
    out = B200Provider()(q.to(DEV), k.to(DEV), v.to(DEV), AttentionOptions(softmax_scale=.13))
    torch.testing.assert_close(out.float().cpu(), oracle.sdpa_fp32(q, k, v, .13), atol=7e-3, rtol=7e-3)


def test_provider_nan_is_not_hidden(cuda_lib):
    from powershard_b200.provider import B200Provider
    q = torch.randn(1, 64, 1, 128, device=DEV, dtype=torch.bfloat16)
    q[0, 1, 0, 0] = float("nan")
    out = B200Provider()(q, q, q)
    assert torch.isnan(out).any()


def test_probe_passes(cuda_lib):
    from powershard_b200.probe import probe
    result = probe()
    assert result["status"] == "PASS" and result["causal"] == "UnsupportedAttention"


# ---------------------------------------------------------------- whole block
@pytest.mark.parametrize("total,heads", [(300, 4), (1023, 3)])
def test_engine_world1_matches_oracle(cuda_lib, oracle, total, heads):
    from powershard_b200.ulysses import UlyssesAttention
    x, wq, wk, freqs = rank_inputs(oracle, total, heads, 7, torch.bfloat16)
    engine = UlyssesAttention()
    out = engine.forward(*(t[0].to(DEV) for t in x), wq.to(DEV), wk.to(DEV), freqs[0, :, 0].to(DEV),
                         total=total, heads=heads, local=True)
    engine.check()
    ref = oracle.sequence_attention(x[0], x[1], x[2], wq, wk, freqs, heads, world=1)[0][0]
    assert_attention_close(out, ref)


@pytest.mark.parametrize("total,heads,world", [(41, 5, 2), (300, 7, 3), (129, 40, 8), (9, 3, 4)])
def test_emulated_ranks_on_one_gpu(cuda_lib, oracle, total, heads, world):
    """The multi-rank data path on one device: per-rank pre-pass, the
    all-to-all done as a device permutation, per-rank attention, the
    inverse permutation and per-rank unpack."""
    from powershard_b200 import ops
    x, wq, wk, freqs = rank_inputs(oracle, total, heads, 9, torch.bfloat16)
    geos = [geometry(total, heads, world, r) for r in range(world)]
    sends = []
    for geo in geos:
        a, b = geo.bounds
        send = torch.empty(geo.send_shape(), dtype=torch.bfloat16, device=DEV)
        ops.prepass(*(t[0, a:b].to(DEV) for t in x), wq.to(DEV), wk.to(DEV), freqs[0, a:b, 0].to(DEV), send, geo)
        sends.append(send)
    recvs = [torch.stack([sends[s][r] for s in range(world)]).contiguous() for r in range(world)]
    outs = []
    for r, geo in enumerate(geos):
        o = torch.zeros(geo.out_shape(), dtype=torch.bfloat16, device=DEV)
        ops.ulysses_attention(recvs[r], o, geo, 128 ** -0.5, None)
        outs.append(o)
    backs = [torch.stack([outs[s][r] for s in range(world)]).contiguous() for r in range(world)]
    expected = oracle.sequence_attention(x[0], x[1], x[2], wq, wk, freqs, heads, world=world)
    for r, geo in enumerate(geos):
        out = torch.empty((geo.n_local, heads, 128), dtype=torch.float32, device=DEV)
        ops.unpack(backs[r], out, geo)
        if geo.n_local:
            assert_attention_close(out, expected[r][0])


@pytest.mark.parametrize("index", [0, 1, 2])
def test_engine_matches_reference_recording(cuda_lib, golden_dir, index):
    """The reference's own sequence_attention output (fp32 wire, fp16
    provider, recorded by tests/golden/make_golden.py) vs this path (bf16
    wire) on the same inputs, rank by rank (ranks emulated on one GPU)."""
    from powershard_b200 import ops
    data = torch.load(golden_dir / "sequence_attention.pt", weights_only=False)
    case = data["cases"][index]
    world, total, heads = case["world"], case["total"], case["heads"]
    geos = [geometry(total, heads, world, r) for r in range(world)]
    sends = []
    for geo in geos:
        a, b = geo.bounds
        send = torch.empty(geo.send_shape(), dtype=torch.bfloat16, device=DEV)
        ops.prepass(*(t[0, a:b].to(torch.bfloat16).to(DEV) for t in (data["q_lin"], data["k_lin"], data["v_lin"])),
                    data["wq"].to(DEV), data["wk"].to(DEV), data["freqs"][0, a:b, 0].to(DEV), send, geo, data["eps"])
        sends.append(send)
    recvs = [torch.stack([sends[s][r] for s in range(world)]).contiguous() for r in range(world)]
    outs = []
    for r, geo in enumerate(geos):
        o = torch.zeros(geo.out_shape(), dtype=torch.bfloat16, device=DEV)
        ops.ulysses_attention(recvs[r], o, geo, 128 ** -0.5, None)
        outs.append(o)
    backs = [torch.stack([outs[s][r] for s in range(world)]).contiguous() for r in range(world)]
    for r, geo in enumerate(geos):
        out = torch.empty((geo.n_local, heads, 128), dtype=torch.float32, device=DEV)
        ops.unpack(backs[r], out, geo)
        assert_attention_close(out, case["ranks"][r]["out"][0])


def test_wan14b_full_size_sampled_rows(cuda_lib, oracle):
    """configs[1] (L=32760, H=40, D=128) at world size 1: sampled query rows
    of sampled heads against the fp32 oracle over all 32760 keys."""
    from powershard_b200.ulysses import UlyssesAttention
    total, heads, grid = 32760, 40, (21, 30, 52)
    g = torch.Generator(device=DEV).manual_seed(0)
    x = [torch.randn(total, heads * 128, device=DEV, generator=g, dtype=torch.bfloat16) * 1.43 for _ in range(3)]
    w = torch.ones(heads * 128, device=DEV)
    freqs = oracle.rope_table_3d(grid, 128)
    engine = UlyssesAttention()
    out = engine.forward(*x, w, w, freqs[0, :, 0].to(DEV), total=total, heads=heads, local=True)
    engine.check()
    rows = torch.tensor([0, 1, 127, 128, 4095, 16383, 20000, 32639, 32640, 32759])
    ones = torch.ones(heads * 128)
    xq, xk, xv = (t.cpu()[None] for t in x)
    q_all = oracle.rms_norm(xq, ones, 1e-6)          # RMSNorm over the full 5120 width
    k_all = oracle.rms_norm(xk, ones, 1e-6)
    for head in (0, 17, 39):
        sl = slice(head * 128, (head + 1) * 128)
        q = oracle.rope_apply(q_all[..., sl].reshape(1, total, 1, 128), freqs).to(torch.bfloat16)
        k = oracle.rope_apply(k_all[..., sl].reshape(1, total, 1, 128), freqs).to(torch.bfloat16)
        v = xv[..., sl].reshape(1, total, 1, 128)
        ref = oracle.sdpa_fp32(q[:, rows], k, v)[0, :, 0]
        assert_attention_close(out[rows, head], ref)


# ------------------------------------------------------- BASELINE config shapes
def _emulated_block(oracle, x, wq, wk, freqs, total, heads, world):
    """Run the whole block for every rank of `world` on one GPU (device-side
    all-to-all emulation); returns per-rank outputs [n_r, H, D] (fp32)."""
    from powershard_b200 import ops
    geos = [geometry(total, heads, world, r) for r in range(world)]
    sends = []
    for geo in geos:
        a, b = geo.bounds
        send = torch.empty(geo.send_shape(), dtype=torch.bfloat16, device=DEV)
        ops.prepass(*(t[a:b] for t in x), wq, wk, freqs[a:b], send, geo)
        sends.append(send)
    outs = []
    for r, geo in enumerate(geos):
        recv = torch.stack([sends[s][r] for s in range(world)]).contiguous()
        o = torch.zeros(geo.out_shape(), dtype=torch.bfloat16, device=DEV)
        ops.ulysses_attention(recv, o, geo, 128 ** -0.5, None)
        outs.append(o)
        del recv
    del sends
    results = []
    for r, geo in enumerate(geos):
        back = torch.stack([outs[s][r] for s in range(world)]).contiguous()
        out = torch.empty((geo.n_local, heads, 128), dtype=torch.float32, device=DEV)
        ops.unpack(back, out, geo)
        results.append(out)
    return results


def test_config1_wan13b_w2_full(cuda_lib, oracle):
    """configs[0] shape (Wan2.1-1.3B: L=4096 on a 16x16x16 grid, 12 heads), W=2, every row."""
    total, heads, grid = 4096, 12, (16, 16, 16)
    g = torch.Generator().manual_seed(0)
    x = [(torch.randn(1, total, heads * 128, generator=g) * 1.43).to(torch.bfloat16) for _ in range(3)]
    w = torch.ones(heads * 128)
    freqs = oracle.rope_table_3d(grid, 128)
    outs = _emulated_block(oracle, [t[0].to(DEV) for t in x], w.to(DEV), w.to(DEV), freqs[0, :, 0].to(DEV),
                           total, heads, 2)
    expected = oracle.sequence_attention(x[0], x[1], x[2], w, w, freqs, heads, world=2)
    for r in range(2):
        assert_attention_close(outs[r], expected[r][0])


def _sampled_rows_check(oracle, out_rows_fn, x_cpu, freqs, total, heads, rows, head_ids):
    ones = torch.ones(heads * 128)
    q_all = oracle.rms_norm(x_cpu[0][None], ones, 1e-6)
    k_all = oracle.rms_norm(x_cpu[1][None], ones, 1e-6)
    for head in head_ids:
        sl = slice(head * 128, (head + 1) * 128)
        q = oracle.rope_apply(q_all[..., sl].reshape(1, total, 1, 128), freqs).to(torch.bfloat16)
        k = oracle.rope_apply(k_all[..., sl].reshape(1, total, 1, 128), freqs).to(torch.bfloat16)
        v = x_cpu[2][None][..., sl].reshape(1, total, 1, 128)
        ref = oracle.sdpa_fp32(q[:, rows], k, v)[0, :, 0]
        assert_attention_close(out_rows_fn(rows, head), ref)


def test_config3_ti2v5b_full_size_sampled_rows(cuda_lib, oracle):
    """configs[2] shape (TI2V-5B: L=27280 on 31x22x40, 24 heads) at W=1."""
    from powershard_b200.ulysses import UlyssesAttention
    total, heads, grid = 27280, 24, (31, 22, 40)
    g = torch.Generator(device=DEV).manual_seed(5)
    x = [torch.randn(total, heads * 128, device=DEV, generator=g, dtype=torch.bfloat16) * 1.43 for _ in range(3)]
    w = torch.ones(heads * 128, device=DEV)
    freqs = oracle.rope_table_3d(grid, 128)
    engine = UlyssesAttention()
    out = engine.forward(*x, w, w, freqs[0, :, 0].to(DEV), total=total, heads=heads, local=True)
    engine.check()
    rows = torch.tensor([0, 5, 127, 128, 9999, 20000, 27135, 27136, 27279])
    _sampled_rows_check(oracle, lambda r, h: out[r, h], [t.cpu() for t in x], freqs, total, heads, rows, (0, 23))


def test_config4_long_75600_w2_sampled_rows(cuda_lib, oracle):
    """configs[3] shape (L=75600 on 21x45x80, 40 heads) at W=2 (ranks emulated
    on one GPU): key segments of 37800 rows, > 64K tokens per attention."""
    total, heads, grid, world = 75600, 40, (21, 45, 80), 2
    g = torch.Generator(device=DEV).manual_seed(6)
    x = [torch.randn(total, heads * 128, device=DEV, generator=g, dtype=torch.bfloat16) * 1.43 for _ in range(3)]
    w = torch.ones(heads * 128, device=DEV)
    freqs = oracle.rope_table_3d(grid, 128)
    outs = _emulated_block(oracle, x, w, w, freqs[0, :, 0].to(DEV), total, heads, world)
    x_cpu = [t.cpu() for t in x]
    del x
    n0 = outs[0].shape[0]

    def rows_of(r, h):
        r = torch.as_tensor(r)
        return torch.stack([outs[int(i) // n0][int(i) % n0, h] for i in r])
    rows = torch.tensor([0, 1, 37799, 37800, 50000, 75599])
    _sampled_rows_check(oracle, rows_of, x_cpu, freqs, total, heads, rows, (0, 21, 39))


# --------------------------------------------------- Flux joint
def _flux_inputs(oracle, txt_len, grid, heads, seed=8):
    g = torch.Generator().manual_seed(seed)
    n_img = grid[0] * grid[1]
    txt = [(torch.randn(1, txt_len, heads * 128, generator=g) * 1.43).to(torch.bfloat16) for _ in range(3)]
    img = [(torch.randn(1, n_img, heads * 128, generator=g) * 1.43).to(torch.bfloat16) for _ in range(3)]
    wq = torch.rand(128, generator=g) + 0.5
    wk = torch.rand(128, generator=g) + 0.5
    table = oracle.rope_table_flux(txt_len, grid, 128)
    return txt, img, wq, wk, table[:, :txt_len], table[:, txt_len:]


@pytest.mark.parametrize("world,txt_len,grid,heads", [(1, 512, (64, 64), 24), (2, 512, (64, 64), 24),
                                                      (3, 77, (20, 30), 5), (4, 512, (64, 64), 24)])
def test_flux_joint_emulated_ranks(cuda_lib, oracle, world, txt_len, grid, heads):
    """configs[4] (Flux.1-dev: 512 text + 64x64 image tokens, 24 heads): text
    replicated, image rows Ulysses-split; ranks emulated on one GPU."""
    from powershard_b200 import ops
    from powershard_b200.partition import UlyssesGeometry
    txt, img, wq, wk, tf, imf = _flux_inputs(oracle, txt_len, grid, heads)
    total = grid[0] * grid[1]
    expected = oracle.flux_joint_attention(txt, img, wq, wk, tf, imf, heads, world)
    geos = [geometry(total, heads, world, r) for r in range(world)]
    tgeo = UlyssesGeometry.replicated(txt_len, heads, 128, world)
    tsend = torch.empty(tgeo.send_shape(), dtype=torch.bfloat16, device=DEV)
    ops.prepass(*(t[0].to(DEV) for t in txt), wq.to(DEV), wk.to(DEV), tf[0, :, 0].to(DEV), tsend, tgeo,
                norm_rope=ops.NORM_PER_HEAD)
    sends = []
    for geo in geos:
        a, b = geo.bounds
        send = torch.empty(geo.send_shape(), dtype=torch.bfloat16, device=DEV)
        ops.prepass(*(t[0, a:b].to(DEV) for t in img), wq.to(DEV), wk.to(DEV), imf[0, a:b, 0].to(DEV), send, geo,
                    norm_rope=ops.NORM_PER_HEAD)
        sends.append(send)
    outs, touts = [], []
    for r, geo in enumerate(geos):
        recv = torch.stack([sends[s][r] for s in range(world)]).contiguous()
        o = torch.zeros(geo.out_shape(), dtype=torch.bfloat16, device=DEV)
        to = torch.zeros((txt_len, geo.heads_per_rank, 128), dtype=torch.bfloat16, device=DEV)
        ops.ulysses_joint_attention(recv, tsend[r], o, to, geo, 128 ** -0.5, None)
        outs.append(o)
        touts.append(to)
    gathered = torch.stack(touts).contiguous()
    txt_out = torch.empty((txt_len, heads, 128), dtype=torch.float32, device=DEV)
    ops.unpack(gathered, txt_out, tgeo)
    for r, geo in enumerate(geos):
        back = torch.stack([outs[s][r] for s in range(world)]).contiguous()
        out = torch.empty((geo.n_local, heads, 128), dtype=torch.float32, device=DEV)
        ops.unpack(back, out, geo)
        if geo.n_local:
            assert_attention_close(out, expected[r][1])
    assert_attention_close(txt_out, expected[0][0])


def test_flux_joint_engine_world1(cuda_lib, oracle):
    from powershard_b200.ulysses import UlyssesAttention
    txt, img, wq, wk, tf, imf = _flux_inputs(oracle, 512, (64, 64), 24)
    engine = UlyssesAttention()
    t_out, i_out = engine.forward_joint([t[0].to(DEV) for t in txt], [t[0].to(DEV) for t in img], wq.to(DEV),
                                        wk.to(DEV), tf[0, :, 0].to(DEV), imf[0, :, 0].to(DEV), total_img=4096,
                                        heads=24)
    engine.check()
    expected = oracle.flux_joint_attention(txt, img, wq, wk, tf, imf, 24, 1)
    assert_attention_close(t_out, expected[0][0])
    assert_attention_close(i_out, expected[0][1])
