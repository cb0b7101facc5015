"""Pin the CPU oracle to the reference: every oracle function against the
fixtures recorded from ComfyUI-PowerShard itself (tests/golden/make_golden.py).
"""
import pytest
import torch


def load(golden_dir, name):
    return torch.load(golden_dir / name, weights_only=False)


@pytest.mark.parametrize("index", [0, 1])
def test_attention_qkv_matches_reference(oracle, golden_dir, index):
    case = load(golden_dir, "attention_qkv.pt")[index]
    q, k, v = oracle.attention_qkv(case["q_lin"], case["k_lin"], case["v_lin"], case["wq"], case["wk"],
                                   case["freqs"], case["heads"], case["eps"])
    # Same operations in the same order as operations.RMSNorm / rope_apply.
    torch.testing.assert_close(q, case["q"], atol=0, rtol=0)
    torch.testing.assert_close(k, case["k"], atol=0, rtol=0)
    torch.testing.assert_close(v, case["v"], atol=0, rtol=0)
    assert q.dtype == torch.float32 and v.dtype == case["v"].dtype


def test_rope_apply_identity_and_norm(oracle):
    x = torch.randn(1, 6, 2, 128)
    ident = oracle.rope_table_3d((1, 1, 1), 128).expand(1, 6, 1, 64, 2, 2)
    torch.testing.assert_close(oracle.rope_apply(x, ident), x)
    table = oracle.rope_table_3d((2, 1, 3), 128)
    out = oracle.rope_apply(x, table)
    torch.testing.assert_close(out.norm(dim=-1), x.norm(dim=-1), rtol=1e-5, atol=1e-5)


def test_rope_axes_split(oracle):
    assert oracle.rope_axes(128) == (44, 42, 42)


@pytest.mark.parametrize("index", range(8))
def test_ulysses_exchange_lhd_matches_reference(oracle, golden_dir, index):
    case = load(golden_dir, "ulysses_exchange.pt")[index]
    assert case["layout"] == "LHD"
    world, total, heads = case["world"], case["total"], case["heads"]
    sends = []
    for r in range(world):
        a, b = oracle.shard_bounds(total, r, world)
        sends.append(oracle.pack_qkv(case["q"][a:b], case["k"][a:b], case["v"][a:b], total, r, world))
    recvs = oracle.exchange(sends)
    attn_outs = []
    for r in range(world):
        ref = case["ranks"][r]
        q, k, v = oracle.unpack_qkv(recvs[r], total)
        torch.testing.assert_close(q, ref["qg"], atol=0, rtol=0)
        torch.testing.assert_close(k, ref["kg"], atol=0, rtol=0)
        torch.testing.assert_close(v, ref["vg"], atol=0, rtol=0)
        assert ref["padded"] == -(-heads // world) * world
        assert ref["nbytes"] == sends[r].numel() * sends[r].element_size()
        got = oracle.math_attention(q[None], k[None], v[None], None, 3, 5)[0]
        torch.testing.assert_close(got, ref["attn"], atol=1e-6 * float(v.abs().max()), rtol=1e-5)
        attn_outs.append(oracle.pack_out(got, total, world))
    back = oracle.exchange(attn_outs)
    for r in range(world):
        out = oracle.unpack_out(back[r], total, heads, r, world)
        torch.testing.assert_close(out, case["ranks"][r]["out"], atol=1e-6 * float(case["v"].abs().max()),
                                   rtol=1e-5)


@pytest.mark.parametrize("index", [8, 9])
def test_ulysses_exchange_blhd_matches_reference(oracle, golden_dir, index):
    case = load(golden_dir, "ulysses_exchange.pt")[index]
    assert case["layout"] == "BLHD"
    world, total, heads = case["world"], case["total"], case["heads"]
    sends = []
    for r in range(world):
        a, b = oracle.shard_bounds(total, r, world)
        sends.append(oracle.pack_qkv(case["q"][0, a:b], case["k"][0, a:b], case["v"][0, a:b], total, r, world))
    recvs = oracle.exchange(sends)
    outs = []
    for r in range(world):
        q, k, v = oracle.unpack_qkv(recvs[r], total)
        ref = case["ranks"][r]
        torch.testing.assert_close(q, ref["qg"][0], atol=0, rtol=0)
        torch.testing.assert_close(v, ref["vg"][0], atol=0, rtol=0)
        outs.append(oracle.pack_out(q, total, world))
    back = oracle.exchange(outs)
    for r in range(world):
        out = oracle.unpack_out(back[r], total, heads, r, world)
        torch.testing.assert_close(out, case["ranks"][r]["back"][0], atol=0, rtol=0)
        assert case["ranks"][r]["nbytes_out"] == outs[r].numel() * outs[r].element_size()


@pytest.mark.parametrize("index", range(4))
def test_math_attention_matches_reference(oracle, golden_dir, index):
    case = load(golden_dir, "math_attention.pt")[index]
    got = oracle.math_attention(case["q"], case["k"], case["v"], case["scale"], case["query_chunk"],
                                case["key_chunk"])
    # Same tiling and operation order; only BLAS thread partitioning of the
    # fp32 matmuls may differ from the recording run (last-bit effects).
    torch.testing.assert_close(got, case["out"], atol=1e-6, rtol=1e-5)
    # The fp32 SDPA oracle of the north star agrees with the tiled math path.
    torch.testing.assert_close(oracle.sdpa_fp32(case["q"], case["k"], case["v"], case["scale"]), case["out"],
                               atol=1e-5, rtol=1e-4)


@pytest.mark.parametrize("index", range(3))
def test_sequence_attention_matches_reference(oracle, golden_dir, index):
    data = load(golden_dir, "sequence_attention.pt")
    case = data["cases"][index]
    outs = oracle.sequence_attention(data["q_lin"], data["k_lin"], data["v_lin"], data["wq"], data["wk"],
                                     data["freqs"], case["heads"], case["world"], data["eps"],
                                     wire_dtype=torch.float32, attention="math", provider_dtype=torch.float16)
    for r, ref in enumerate(case["ranks"]):
        torch.testing.assert_close(outs[r], ref["out"], atol=1e-6, rtol=1e-5)
        assert ref["counters"]["kv_collectives"] == 1 and ref["counters"]["out_collectives"] == 1


def test_sdpa_oracle_close_to_reference_path(oracle, golden_dir):
    """The fp32 SDPA oracle used for CUDA parity differs from the reference's
    fp16-cast provider path only by the fp16 input rounding."""
    data = load(golden_dir, "sequence_attention.pt")
    case = data["cases"][2]
    outs = oracle.sequence_attention(data["q_lin"], data["k_lin"], data["v_lin"], data["wq"], data["wk"],
                                     data["freqs"], case["heads"], case["world"], data["eps"],
                                     wire_dtype=torch.float32, attention="sdpa")
    for r, ref in enumerate(case["ranks"]):
        err = (outs[r] - ref["out"]).abs()
        assert float(err.max()) < 2e-2
        assert float(err.mean() / ref["out"].abs().mean()) < 5e-3


def test_product_rope_tables_match_oracle(oracle):
    from powershard_b200 import rope
    for grid in ((2, 3, 4), (21, 30, 52)):
        torch.testing.assert_close(rope.rope_table_3d(grid, 128), oracle.rope_table_3d(grid, 128)[0, :, 0])
    torch.testing.assert_close(rope.rope_table_flux(5, (4, 6), 128), oracle.rope_table_flux(5, (4, 6), 128)[0, :, 0])


@pytest.mark.parametrize("index", range(4))
def test_image_sequence_attention_matches_reference(oracle, golden_dir, index):
    """image_parallel.SequenceAttention over image_layout.Layout (balanced
    split of the image segment, replicated text/reference segments)."""
    case = load(golden_dir, "image_sequence_attention.pt")[index]
    world, heads = case["world"], case["heads"]
    q, k, v = (t.transpose(1, 2) for t in (case["q"], case["k"], case["v"]))  # BHLD -> BLHD
    split = [n for n, s in case["segments"] if s][0]
    outs = oracle.image_sequence_attention(q, k, v, case["segments"], world)
    for r, ref in enumerate(case["ranks"]):
        assert oracle.split_sizes(split, world) == ref["sizes"]
        assert oracle.image_local_ranges(case["segments"], world, r) == [tuple(x) for x in ref["local_ranges"]]
        got = outs[r].reshape(outs[r].shape[0], outs[r].shape[1], -1)
        assert got.shape[1] == ref["local_len"]
        torch.testing.assert_close(got, ref["out"], atol=1e-6, rtol=1e-5)
        assert ref["stats"]["attention_calls"] == 1


def test_product_image_layout_matches_oracle(oracle, golden_dir):
    """powershard_b200.partition.ImageLayout / split_sizes and a geometry
    built from the layout agree with the recorded reference Layout."""
    from powershard_b200.partition import ImageLayout, UlyssesGeometry, split_sizes
    for case in load(golden_dir, "image_sequence_attention.pt"):
        world = case["world"]
        split = [n for n, s in case["segments"] if s][0]
        for r, ref in enumerate(case["ranks"]):
            lay = ImageLayout(case["segments"], world, r)
            assert lay.sizes == ref["sizes"] == split_sizes(split, world)
            assert (lay.local_len, lay.chunk) == (ref["local_len"], ref["chunk"])
            geo = UlyssesGeometry(total=split, heads=5, head_dim=128, world=world, rank=r, sizes=lay.sizes)
            assert geo.width == lay.chunk and geo.seg_valid() == lay.sizes
            assert geo.bounds == (lay.a - lay.split_start, lay.b - lay.split_start)


@pytest.mark.parametrize("index", range(3))
def test_token_sequence_attention_matches_reference(oracle, golden_dir, index):
    """sequence_mode="token": K/V all-gathered, local queries (math provider, fp32 wire)."""
    data = load(golden_dir, "sequence_attention_token.pt")
    case = data["cases"][index]
    outs = oracle.token_sequence_attention(data["q_lin"], data["k_lin"], data["v_lin"], data["wq"], data["wk"],
                                           data["freqs"], case["heads"], case["world"], data["eps"],
                                           attention="math", provider_dtype=torch.float16)
    for r, ref in enumerate(case["ranks"]):
        torch.testing.assert_close(outs[r], ref["out"], atol=1e-6, rtol=1e-5)
        assert ref["counters"]["kv_collectives"] == 1 and ref["counters"]["out_collectives"] == 0
        # gathered bytes: the reference gathers [1, total, 2, H, D] in the fp32 wire
        assert ref["counters"]["kv_gathered_bytes"] == 2 * case["total"] * case["heads"] * case["dim"] * 4


@pytest.mark.parametrize("index", range(3))
def test_rope_split_half_matches_reference(oracle, golden_dir, index):
    """H3 partial RoPE (attention.rope_split_half): pairs (j, j+P), tail unrotated."""
    case = load(golden_dir, "rope_split_half.pt")[index]
    got = oracle.rope_split_half(case["x"], case["table"])
    assert got.dtype == case["out"].dtype
    # Separate multiply and add per element vs the reference's 2x2 matmul: at
    # most one fp32 rounding apart before the cast.
    if case["x"].dtype == torch.float32:
        torch.testing.assert_close(got, case["out"], atol=1e-6, rtol=1e-6)
    else:
        diff = (got.float() - case["out"].float()).abs()
        assert float((diff > 0).float().mean()) < 0.01
        assert float(diff.max()) <= float(case["out"].float().abs().max()) * 2 ** -7
    p = case["table"].shape[-3]
    assert torch.equal(got[..., 2 * p:], case["x"][..., 2 * p:])


@pytest.mark.parametrize("index", range(2))
def test_self_attention_forward_batch2_matches_reference(oracle, golden_dir, index):
    """wan_model.self_attention_forward on a CFG batch of 2 (q/k/v/o Linear with
    bias, attention_qkv, sequence_attention, o) restated with the oracle,
    one batch row at a time, against the reference's recording (W = 1 with
    the sequence state off, W = 2 Ulysses); the recorded counters count the
    whole batch in one exchange, fp32 wire."""
    import torch.nn.functional as F
    data = load(golden_dir, "self_attention_forward.pt")
    case = data["cases"][index]
    world, heads = case["world"], data["heads"]
    x = data["x"]
    batch, total, hidden = x.shape
    # Projections per rank shard, as each rank of the reference computes them
    # (the BLAS blocking of a shard differs from that of the whole sequence).
    bounds = [oracle.shard_bounds(total, r, world) for r in range(world)]
    lin = [torch.cat([F.linear(x[:, a:z], w, b) for a, z in bounds], dim=1)
           for w, b in zip(data["weights"][:3], data["biases"][:3])]
    # The reference's power-of-two V scale covers the whole batch a rank receives.
    h = -(-heads // world)
    v_all = lin[2].view(batch, total, heads, -1)
    v_scales = [oracle._power2_scale(v_all[:, :, r * h:(r + 1) * h].abs().amax() / 16384.0)
                for r in range(world)]
    rows = []
    for b in range(batch):
        outs = oracle.sequence_attention(lin[0][b:b + 1], lin[1][b:b + 1], lin[2][b:b + 1], data["wq"], data["wk"],
                                         data["freqs"], heads, world, data["eps"], wire_dtype=torch.float32,
                                         attention="math", provider_dtype=torch.float16, v_scales=v_scales)
        rows.append(outs)
    for r, ref in enumerate(case["ranks"]):
        a, bnd = ref["bounds"]
        attn = torch.cat([rows[b][r] for b in range(batch)]).reshape(batch, bnd - a, hidden)
        out = F.linear(attn, data["weights"][3], data["biases"][3])
        torch.testing.assert_close(out, ref["out"], atol=2e-6, rtol=1e-5)
        if world > 1:
            width, h = -(-total // world), -(-heads // world)
            c = ref["counters"]
            assert c["kv_collectives"] == 1 and c["out_collectives"] == 1
            assert c["kv_gathered_bytes"] == world * 3 * batch * width * h * 128 * 4
            assert c["out_exchanged_bytes"] == world * batch * width * h * 128 * 4
