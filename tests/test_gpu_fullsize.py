"""Every row and head of the BASELINE headline configs, and the Wan / LTX
entry points, on the CUDA path (needs a B200).

The full-size reference is ``fp32_attention``: softmax(Q K^T * scale) V in
fp32 on the device, a few hundred query rows at a time (TF32 off), applied
to the fp32 restatement of the pre-pass (RMSNorm over the full width,
rounded to the projection dtype as the reference's RMSNorm returns it, then
RoPE in fp32 and the bf16 wire).  ``test_fp32_reference_matches_oracle``
pins that device reference to the CPU oracle on a small case.

Tolerance (the north star's): max |err| <= 2e-2 and mean |err| / mean |ref|
<= 5e-3 over the whole output tensor.
"""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
MAX_ABS, MEAN_REL = 2e-2, 5e-3


def assert_close_full(got, ref, max_abs=MAX_ABS, mean_rel=MEAN_REL):
    """Whole-tensor error statistics, computed on the device."""
    assert got.shape == ref.shape, (got.shape, ref.shape)
    got = got.float()
    assert bool(torch.isfinite(got).all())
    err = (got - ref).abs()
    m = float(err.max())
    rel = float(err.double().sum() / ref.abs().double().sum().clamp_min(1e-30))
    assert m <= max_abs and rel <= mean_rel, f"max_abs={m:.3e} mean_rel={rel:.3e}"
    return m, rel


def fp32_attention(q, k, v, scale=None, rows=256):
    """q [Lq, H, D], k/v [Lk, H, D] (any float dtype) -> [Lq, H, D] fp32 on the
    device: exact softmax attention, `rows` query rows per step."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        scale = q.shape[-1] ** -0.5 if scale is None else scale
        kt = k.float().permute(1, 2, 0).contiguous()   # [H, D, Lk]
        vh = v.float().permute(1, 0, 2).contiguous()   # [H, Lk, D]
        out = torch.empty(q.shape, dtype=torch.float32, device=q.device)
        for a in range(0, q.shape[0], rows):
            qs = q[a:a + rows].float().permute(1, 0, 2)  # [H, r, D]
            s = torch.bmm(qs, kt).mul_(scale)
            s = torch.softmax(s, dim=-1)
            out[a:a + rows] = torch.bmm(s, vh).permute(1, 0, 2)
            del s
        return out
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def prepass_fp32(x, w, table, heads, eps=1e-6, wire=torch.bfloat16):
    """fp32 restatement of RMSNorm (full width, rounded to x.dtype) + interleaved
    RoPE, cast to the wire dtype: x [L, H*D], table [L, D/2, 2, 2] -> [L, H, D]."""
    xf = x.float()
    y = (xf * torch.rsqrt(xf.square().mean(-1, keepdim=True) + eps) * w.float()).to(x.dtype).float()
    y = y.view(x.shape[0], heads, -1, 1, 2)
    rot = table[:, None]
    return (rot[..., 0] * y[..., 0] + rot[..., 1] * y[..., 1]).reshape(x.shape[0], heads, -1).to(wire)


def _grid_table(grid, device):
    from powershard_b200.rope import rope_table_3d
    return rope_table_3d(grid, 128, device=device)


def test_fp32_reference_matches_oracle(cuda_lib, oracle):
    heads, grid = 3, (3, 7, 11)
    total = math.prod(grid)
    g = torch.Generator().manual_seed(4)
    x = [(torch.randn(total, heads * 128, generator=g) * 1.4).to(torch.bfloat16) for _ in range(3)]
    w = (torch.rand(heads * 128, generator=g) + 0.5)
    table = oracle.rope_table_3d(grid, 128)
    q, k, v = oracle.attention_qkv(x[0][None], x[1][None], x[2][None], w, w, table, heads)
    ref = oracle.sdpa_fp32(q.to(torch.bfloat16), k.to(torch.bfloat16), v.to(torch.bfloat16))[0]
    tab = table[0, :, 0].to(DEV)
    qd, kd = (prepass_fp32(t.to(DEV), w.to(DEV), tab, heads) for t in x[:2])
    got = fp32_attention(qd, kd, x[2].to(DEV).view(total, heads, 128), rows=50)
    torch.testing.assert_close(got.cpu(), ref, atol=2e-5, rtol=1e-4)


def _inputs(total, heads, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return [torch.randn(total, heads * 128, device=DEV, generator=g, dtype=torch.bfloat16) * 1.43
            for _ in range(3)]


def test_config1_wan14b_every_row_w1(cuda_lib):
    """configs[1] (L=32760 on 21x30x52, 40 heads) at world size 1: all
    32760 x 40 output rows against the fp32 reference."""
    from powershard_b200.ulysses import UlyssesAttention
    total, heads, grid = 32760, 40, (21, 30, 52)
    x = _inputs(total, heads, 0)
    w = torch.ones(heads * 128, device=DEV)
    table = _grid_table(grid, DEV)
    engine = UlyssesAttention()
    out = engine.forward(*x, w, w, table, total=total, heads=heads, local=True)
    engine.check()
    q, k = (prepass_fp32(t, w, table, heads) for t in x[:2])
    ref = fp32_attention(q, k, x[2].view(total, heads, 128))
    del q, k
    assert_close_full(out, ref)


def test_config3_long_75600_every_row_w2(cuda_lib):
    """configs[3] (L=75600 on 21x45x80, 40 heads) at W=2, ranks emulated on
    one GPU (pre-pass per rank, the all-to-all as a device permutation,
    attention per rank, the inverse permutation, unpack): every row and head
    against the fp32 reference."""
    from powershard_b200 import ops
    from powershard_b200.partition import UlyssesGeometry
    total, heads, grid, world = 75600, 40, (21, 45, 80), 2
    x = _inputs(total, heads, 6)
    w = torch.ones(heads * 128, device=DEV)
    table = _grid_table(grid, DEV)
    geos = [UlyssesGeometry(total=total, heads=heads, head_dim=128, world=world, rank=r) for r in range(world)]
    sends = []
    for geo in geos:
        a, b = geo.bounds
        send = torch.empty(geo.send_shape(), dtype=torch.bfloat16, device=DEV)
        ops.prepass(*(t[a:b] for t in x), w, w, table[a:b], send, geo)
        sends.append(send)
    outs = []
    ws = ops.attention_workspace(DEV)
    for r, geo in enumerate(geos):
        recv = torch.stack([sends[s][r] for s in range(world)]).contiguous()
        o = torch.zeros(geo.out_shape(), dtype=torch.bfloat16, device=DEV)
        ops.ulysses_attention(recv, o, geo, 128 ** -0.5, None, workspace=ws)
        outs.append(o)
        del recv
    del sends
    full = []
    for r, geo in enumerate(geos):
        back = torch.stack([outs[s][r] for s in range(world)]).contiguous()
        out = torch.empty((geo.n_local, heads, 128), dtype=torch.bfloat16, device=DEV)
        ops.unpack(back, out, geo)
        full.append(out)
    del outs
    got = torch.cat(full)
    q, k = (prepass_fp32(t, w, table, heads) for t in x[:2])
    ref = fp32_attention(q, k, x[2].view(total, heads, 128), rows=128)
    del q, k
    assert_close_full(got, ref)


def test_engine_batch_matches_fp32(cuda_lib):
    """forward_batch (one pre-pass, one attention launch, one exchange for the
    whole batch) against the fp32 reference of each batch row, at W=1 and
    with ranks emulated at W=2 and 3; one exchange counted per call.  (The
    batched and row-by-row launches split their last wave differently, so
    their bf16 outputs differ at the kernel's own error level; each is
    compared with the fp32 reference.)"""
    from emulated_dist import emulated_group
    from powershard_b200.partition import shard_bounds
    from powershard_b200.ulysses import UlyssesAttention
    total, heads, batch = 1000, 5, 2
    g = torch.Generator(device=DEV).manual_seed(12)
    x = [torch.randn(batch, total, heads * 128, device=DEV, generator=g, dtype=torch.bfloat16) for _ in range(3)]
    w = torch.rand(heads * 128, device=DEV, generator=g) + 0.5
    table = _grid_table((10, 10, 10), DEV)
    ref = torch.stack([fp32_attention(prepass_fp32(x[0][b], w, table, heads), prepass_fp32(x[1][b], w, table, heads),
                                      x[2][b].view(total, heads, 128)) for b in range(batch)])
    for world in (1, 2, 3):
        def rank_fn(rank):
            a, b = shard_bounds(total, rank, world)
            engine = UlyssesAttention()
            state = {}
            got = engine.forward_batch(*(t[:, a:b] for t in x), w, w, table[a:b], total=total, heads=heads,
                                       state=state)
            engine.check()
            return (a, b), got, state
        if world == 1:
            results = [rank_fn(0)]
        else:
            with emulated_group(world) as run:
                results = run(rank_fn)
        for (a, b), got, state in results:
            assert got.shape == (batch, b - a, heads, 128)
            if b > a:
                assert_close_full(got, ref[:, a:b])
            assert state["kv_collectives"] == 1 and state["out_collectives"] == 1


def _wan_module(data, heads):
    hidden = data["x"].shape[-1]
    module = torch.nn.Module()
    for name, w, bias in zip("qkvo", data["weights"], data["biases"]):
        lin = torch.nn.Linear(hidden, hidden)
        lin.weight.data.copy_(w)
        lin.bias.data.copy_(bias)
        setattr(module, name, lin)
    module.norm_q = torch.nn.RMSNorm(hidden, eps=data["eps"])
    module.norm_k = torch.nn.RMSNorm(hidden, eps=data["eps"])
    module.norm_q.weight.data.copy_(data["wq"])
    module.norm_k.weight.data.copy_(data["wk"])
    module.num_heads, module.head_dim = heads, hidden // heads
    return module.to(DEV)


def test_self_attention_forward_cfg_batch_matches_reference(cuda_lib, golden_dir):
    """wan.self_attention_forward, the hook install_wan_compute sets
    (powershard/wan_model.py:433-438), on a CFG batch of 2 rows with q/k/v/o
    Linear layers (bias) and RMSNorm weights: the reference's own recorded
    output (fp32 Linear, fp16 math provider) against this path (bf16 wire),
    sequence state off (W = 1) and on (Ulysses over one rank)."""
    data = torch.load(golden_dir / "self_attention_forward.pt", weights_only=False)
    heads = data["heads"]
    ref = data["cases"][0]["ranks"][0]["out"].to(DEV)
    x, freqs = data["x"].to(DEV), data["freqs"].to(DEV)
    for enabled in (False, True):
        from powershard_b200 import wan
        module = _wan_module(data, heads)
        module._ps_sequence = dict(total=x.shape[1], enabled=enabled, ulysses=True, comm_dtype="bf16")
        with torch.no_grad():
            out = wan.self_attention_forward(module, x, freqs)
        module._ps_b200_engine.check()
        assert out.shape == ref.shape and out.dtype == torch.float32
        assert_close_full(out, ref)
        if enabled:
            st = module._ps_sequence
            assert st["kv_collectives"] == 1 and st["out_collectives"] == 1
            assert st["kv_gathered_bytes"] == 3 * 2 * x.shape[1] * heads * 128 * 2  # bf16 wire, both rows


def test_ltx_video_self_attention_shape(cuda_lib, oracle):
    """LTX video self-attention (powershard/ltx_model.py:281-296) calls
    sequence_attention(attn, q, k, v) with q/k already rotated in fp32 and
    the module's ``heads``/``dim_head`` (install copies them to num_heads /
    head_dim, ltx_model.py:538-547): an LTX-2-shaped call (32 heads x 128,
    CFG batch 2) with the state off and on."""
    from powershard_b200 import wan
    batch, n, heads = 2, 1200, 32
    g = torch.Generator().manual_seed(21)
    q, k, v = (torch.randn(batch, n, heads, 128, generator=g) for _ in range(3))
    ref = torch.cat([oracle.sdpa_fp32(q[b:b + 1].bfloat16(), k[b:b + 1].bfloat16(), v[b:b + 1].bfloat16())
                     for b in range(batch)])
    for enabled in (False, True):
        attn = type("LTXAttention", (), {})()
        attn.heads, attn.dim_head = heads, 128
        attn.num_heads, attn.head_dim = attn.heads, attn.dim_head
        attn._ps_sequence = dict(total=n, enabled=enabled, ulysses=True, comm_dtype="bf16")
        out = wan.sequence_attention(attn, q.to(DEV), k.to(DEV), v.to(DEV))
        assert out.dtype == torch.float32 and out.shape == (batch, n, heads, 128)
        assert_close_full(out, ref.to(DEV))
