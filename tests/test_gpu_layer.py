"""The whole self-attention layer in the fused kernels (needs a B200):
UlyssesAttention.forward_layer - q/k/v GEMM with RMSNorm + RoPE + pack in
its epilogue, attention, output GEMM reading the exchange buffer in place -
against a plain PyTorch fp32 restatement of the reference's layer
(powershard/wan_model.py:421-438: Linear q/k/v, RMSNorm over the full width,
rope_apply, softmax attention, Linear o).

Tolerance: the north-star bound on the attention output, applied to the
layer output divided by the o-projection's gain - max |err| <= 2e-2 * g and
mean |err| / mean |ref| <= 5e-3, g = the largest absolute row sum of W_o.
"""
import pytest
import torch

from test_gpu_fullsize import fp32_attention

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def layer_reference(x, ws, bs, nq, nk, table, heads, eps=1e-6):
    """fp32 layer for one batch row: x [n, hidden] -> [n, out]."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        xf = x.float()
        q, k, v = (xf @ w.float().t() + (0 if b is None else b.float()) for w, b in zip(ws[:3], bs[:3]))

        def norm_rope(y, w):
            y = y * torch.rsqrt(y.square().mean(-1, keepdim=True) + eps) * w.float()
            y = y.view(y.shape[0], heads, -1, 1, 2)
            rot = table[:, None]
            return (rot[..., 0] * y[..., 0] + rot[..., 1] * y[..., 1]).reshape(y.shape[0], heads, -1)
        o = fp32_attention(norm_rope(q, nq), norm_rope(k, nk), v.view(v.shape[0], heads, -1))
        out = o.reshape(o.shape[0], -1) @ ws[3].float().t()
        return out if bs[3] is None else out + bs[3].float()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def assert_layer_close(got, ref, w_o):
    gain = float(w_o.float().abs().sum(1).max())
    err = (got.float() - ref).abs()
    m = float(err.max())
    rel = float(err.double().sum() / ref.abs().double().sum())
    assert m <= 2e-2 * gain and rel <= 5e-3, f"max_abs={m:.3e} (bound {2e-2 * gain:.3e}) mean_rel={rel:.3e}"


def _layer_inputs(total, heads, fin, fout, batch, seed, bias=True):
    from powershard_b200.rope import rope_table_3d
    d = 128
    g = torch.Generator(device=DEV).manual_seed(seed)
    x = torch.randn(batch, total, fin, device=DEV, generator=g).bfloat16()
    ws = [(torch.randn(heads * d, fin, device=DEV, generator=g) * 0.02).bfloat16() for _ in range(3)]
    ws.append((torch.randn(fout, heads * d, device=DEV, generator=g) * 0.02).bfloat16())
    bs = [torch.randn(n, device=DEV, generator=g) * 0.02 if bias else None for n in (heads * d,) * 3 + (fout,)]
    nq = torch.rand(heads * d, device=DEV, generator=g) + 0.5
    nk = torch.rand(heads * d, device=DEV, generator=g) + 0.5
    side = 12
    table = rope_table_3d((total // (side * side) + 1, side, side), d, device=DEV)[:total].contiguous()
    return x, ws, bs, nq, nk, table


@pytest.mark.parametrize("world", [1, 2, 3])
def test_forward_layer_matches_fp32_layer(cuda_lib, world):
    """CFG batch of 2, biases on every Linear; ranks emulated on one GPU for
    W > 1 (the NCCL exchange over device copies)."""
    from emulated_dist import emulated_group
    from powershard_b200.partition import shard_bounds
    from powershard_b200.ulysses import UlyssesAttention
    total, heads, fin, fout, batch = 1000, 6, 768, 768, 2
    x, ws, bs, nq, nk, table = _layer_inputs(total, heads, fin, fout, batch, 7)
    refs = [layer_reference(x[b], ws, bs, nq, nk, table, heads) for b in range(batch)]

    def rank_fn(rank):
        a, b = shard_bounds(total, rank, world)
        engine = UlyssesAttention()
        state = {}
        out = engine.forward_layer(x[:, a:b].contiguous(), *ws, nq, nk, table[a:b], *bs, total=total, heads=heads,
                                   out_dtype=torch.float32, state=state, local=world == 1)
        engine.check()
        return (a, b), out, state
    if world == 1:
        results = [rank_fn(0)]
    else:
        with emulated_group(world) as run:
            results = run(rank_fn)
    for (a, b), out, state in results:
        for r in range(batch):
            if b > a:
                assert_layer_close(out[r], refs[r][a:b], ws[3])
        assert state["kv_collectives"] == 1


def test_wan_hook_fused_and_unfused_agree(cuda_lib):
    """wan.self_attention_forward with plain bf16 Linear layers runs the fused
    layer; with fused projections switched off it runs the module's own
    Linear layers and the pre-pass.  Both agree with the fp32 layer."""
    from powershard_b200 import wan
    total, heads, fin = 800, 4, 512
    x, ws, bs, nq, nk, table = _layer_inputs(total, heads, fin, fin, 2, 11)
    module = torch.nn.Module()
    for name, w, b in zip("qkvo", ws, bs):
        lin = torch.nn.Linear(w.shape[1], w.shape[0], device=DEV, dtype=torch.bfloat16)
        lin.weight.data.copy_(w)
        lin.bias.data.copy_(b)
        setattr(module, name, lin)
    module.norm_q = torch.nn.RMSNorm(heads * 128, eps=1e-6, device=DEV)
    module.norm_k = torch.nn.RMSNorm(heads * 128, eps=1e-6, device=DEV)
    module.norm_q.weight.data.copy_(nq)
    module.norm_k.weight.data.copy_(nk)
    module.num_heads, module.head_dim = heads, 128
    freqs = table[None, :, None]
    bs = [b.bfloat16().float() for b in bs]  # the bf16 Linear layers hold bf16 biases
    outs = {}
    for fused in (True, False):
        module._ps_b200_fused_projections = fused
        module.__dict__.pop("_ps_b200_fused_cache", None)
        module._ps_sequence = dict(total=total, enabled=False, ulysses=True, comm_dtype="bf16")
        with torch.no_grad():
            outs[fused] = wan.self_attention_forward(module, x, freqs)
        module._ps_b200_engine.check()
        assert (getattr(module, "_ps_b200_fused_cache", None) is not None) == fused
    for r in range(2):
        ref = layer_reference(x[r], ws, bs, nq, nk, table, heads)
        for fused in (True, False):
            assert_layer_close(outs[fused][r], ref, ws[3])


def test_config1_layer_every_row(cuda_lib):
    """configs[1] (L=32760 on 21x30x52, 40 heads x 128, hidden 5120) at W=1:
    the fused layer against the fp32 layer on every row."""
    from powershard_b200.rope import rope_table_3d
    from powershard_b200.ulysses import UlyssesAttention
    total, heads, fin = 32760, 40, 5120
    g = torch.Generator(device=DEV).manual_seed(0)
    x = torch.randn(1, total, fin, device=DEV, generator=g).bfloat16()
    ws = [(torch.randn(heads * 128, fin, device=DEV, generator=g) * 0.02).bfloat16() for _ in range(4)]
    ones = torch.ones(heads * 128, device=DEV)
    table = rope_table_3d((21, 30, 52), 128, device=DEV)
    engine = UlyssesAttention()
    out = engine.forward_layer(x, *ws, ones, ones, table, total=total, heads=heads, out_dtype=torch.float32,
                               local=True)
    engine.check()
    ref = layer_reference(x[0], ws, [None] * 4, ones, ones, table, heads)
    assert_layer_close(out[0], ref, ws[3])
