"""H3 (MiniMax) attention on the CUDA path (needs a B200).

Per-head RMSNorm + split-half partial RoPE (attention.py:98-103, pinned by
tests/golden/rope_split_half.pt) fused into the pre-pass, then the Ulysses
or token exchange, against the oracle.  Pre-pass: each element within 2
16-bit ulps of the oracle, >= 99 % bit-identical; blocks: max |err| <= 2e-2,
mean |err| / mean |ref| <= 5e-3.
"""
from types import SimpleNamespace

import pytest
import torch
from emulated_dist import emulated_group

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def assert_attention_close(got, ref, max_abs=2e-2, mean_rel=5e-3):
    got, ref = got.float().cpu(), ref.float().cpu()
    assert got.shape == ref.shape
    assert torch.isfinite(got).all()
    err = (got - ref).abs()
    rel = float(err.mean() / ref.abs().mean().clamp_min(1e-12))
    assert float(err.max()) <= max_abs and rel <= mean_rel, f"max_abs={float(err.max()):.3e} mean_rel={rel:.3e}"


def split_table(n, pairs, seed):
    g = torch.Generator().manual_seed(seed)
    ang = torch.rand(n, pairs, generator=g, dtype=torch.float64) * 30.0
    c, s = torch.cos(ang), torch.sin(ang)
    return torch.stack([c, -s, s, c], -1).reshape(1, n, 1, pairs, 2, 2).float()


def oracle_qkv(oracle, qkv, wq, wk, table, heads, eps=1e-6):
    """Per-head RMSNorm + rope_split_half of the fused projection [n, 3*H*D]."""
    n = qkv.shape[0]
    q, k, v = qkv.float().to(torch.bfloat16).split(heads * 128, dim=-1)
    qn = oracle.rms_norm_heads(q[None], wq, heads, eps)[0]
    kn = oracle.rms_norm_heads(k[None], wk, heads, eps)[0]
    return (oracle.rope_split_half(qn, table), oracle.rope_split_half(kn, table),
            v.reshape(n, heads, 128))


@pytest.mark.parametrize("n,heads,world,pairs", [(77, 4, 1, 32), (300, 6, 3, 64), (130, 3, 2, 16)])
def test_prepass_split_half_matches_oracle(cuda_lib, oracle, n, heads, world, pairs):
    from powershard_b200 import ops
    from powershard_b200.partition import UlyssesGeometry
    g = torch.Generator().manual_seed(n)
    qkv = (torch.randn(n, 3 * heads * 128, generator=g) * 1.3).bfloat16()
    wq = (torch.rand(128, generator=g) + 0.5).bfloat16()
    wk = (torch.rand(128, generator=g) + 0.5).bfloat16()
    table = split_table(n, pairs, 5)
    q_ref, k_ref, v_ref = oracle_qkv(oracle, qkv, wq, wk, table, heads)
    geo = UlyssesGeometry(total=n * world, heads=heads, head_dim=128, world=world, rank=0)
    send = torch.empty(geo.send_shape(), dtype=torch.bfloat16, device=DEV)
    x = qkv.to(DEV)
    views = [t.view(n, heads, 128) for t in x.split(heads * 128, dim=-1)]
    ops.prepass(*views, wq.to(DEV), wk.to(DEV), table[0, :, 0].contiguous().to(DEV), send, geo,
                norm_rope=ops.NORM_PER_HEAD, rope_split_pairs=pairs)
    torch.cuda.synchronize()
    got = send.cpu()
    h = geo.heads_per_rank
    for kind, ref in enumerate((q_ref, k_ref, v_ref)):
        full = torch.zeros(n, world * h, 128, dtype=torch.bfloat16)
        full[:, :heads] = ref
        mine = got[:, kind, :n].permute(1, 0, 2, 3).reshape(n, world * h, 128)
        diff = (mine.float() - full.float()).abs()
        ulp = full.float().abs().clamp_min(2 ** -20) * 2 ** -7
        assert bool((diff <= 2 * ulp).all()), kind
        assert float((mine == full).float().mean()) >= 0.99, kind
        assert not got[:, kind, n:].any()


class _Linear:
    def __init__(self, w):
        self.w = w

    def __call__(self, x):
        return x @ self.w.t()


def _module(heads, wq, wk, proj):
    return SimpleNamespace(heads=heads, head_dim=128, qkv_proj=_Linear(proj),
                           q_norm=SimpleNamespace(weight=wq, eps=1e-6), k_norm=SimpleNamespace(weight=wk, eps=1e-6),
                           out_proj=lambda t: t)


@pytest.mark.parametrize("total,heads,world,ulysses,pairs", [(500, 4, 1, True, 32), (1000, 6, 2, True, 64),
                                                             (517, 5, 3, True, 32), (700, 4, 2, False, 16)])
def test_h3_attention_forward_matches_oracle(cuda_lib, oracle, total, heads, world, ulysses, pairs):
    from powershard_b200 import h3
    import types
    g = torch.Generator().manual_seed(total)
    dim = 256
    x = (torch.randn(total, dim, generator=g)).bfloat16()
    proj = (torch.randn(3 * heads * 128, dim, generator=g) * 0.08).bfloat16()
    wq = (torch.rand(128, generator=g) + 0.5).bfloat16()
    wk = (torch.rand(128, generator=g) + 0.5).bfloat16()
    table = split_table(total, pairs, 6)
    q, k, v = oracle_qkv(oracle, (x.float() @ proj.float().t()).bfloat16(), wq, wk, table, heads)
    ref = oracle.sdpa_fp32(q.float()[None], k.float()[None], v.float()[None])[0]   # [total, H, D]

    def rank_fn(rank):
        a, b = oracle.shard_bounds(total, rank, world)
        m = _module(heads, wq.to(DEV), wk.to(DEV), proj.to(DEV))
        m.forward = types.MethodType(h3.attention_forward, m)
        m._ps_sequence = dict(total=total, enabled=world > 1, ulysses=ulysses, comm_dtype="bf16")
        out = m.forward(x[a:b].to(DEV), table[:, a:b].to(DEV))
        m._ps_b200_engine.check()
        return (a, b), out.cpu()

    if world == 1:
        outs = [rank_fn(0)]
    else:
        with emulated_group(world) as run:
            outs = run(rank_fn)
    for (a, b), out in outs:
        if b > a:
            assert_attention_close(out.reshape(b - a, heads, 128), ref[a:b])
