"""Token mode (the reference's sequence_mode="token") on the CUDA path (needs a B200).

One K/V all-gather per block, queries local, attention of the rank's rows
against every rank's keys written straight to the output
(powershard/wan_model.py:489-500).  Checked against the oracle's
restatement, which is pinned to the reference's recorded token-mode outputs;
W > 1 runs as threads on one GPU with in-process collectives.  Tolerance:
max |err| <= 2e-2 and mean |err| / mean |ref| <= 5e-3.
"""
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


def _inputs(oracle, total, heads, seed=14):
    g = torch.Generator().manual_seed(seed)
    x = [(torch.randn(1, total, heads * 128, generator=g) * 1.5).bfloat16() for _ in range(3)]
    wq = torch.rand(heads * 128, generator=g) + 0.5
    wk = torch.rand(heads * 128, generator=g) + 0.5
    freqs = oracle.rope_table_3d((total // 100 + 1, 10, 10), 128)[:, :total]
    return x, wq, wk, freqs


@pytest.mark.parametrize("total,heads,world", [(300, 4, 1), (1023, 3, 1), (1000, 40, 2), (41, 5, 3), (4099, 6, 4),
                                               (9, 3, 4)])
def test_token_mode_matches_oracle(cuda_lib, oracle, total, heads, world):
    from powershard_b200.ulysses import UlyssesAttention
    x, wq, wk, freqs = _inputs(oracle, total, heads)
    expected = oracle.token_sequence_attention(*(t.float() for t in x), wq, wk, freqs, heads, world)

    def rank_fn(rank):
        a, b = oracle.shard_bounds(total, rank, world)
        engine = UlyssesAttention()
        state = {}
        out = engine.forward_token(*(t[0, a:b].to(DEV) for t in x), wq.to(DEV), wk.to(DEV),
                                   freqs[0, a:b, 0].to(DEV), total=total, heads=heads, state=state)
        engine.check()
        assert state["kv_collectives"] == 1
        return out.cpu()

    if world == 1:
        outs = [rank_fn(0)]
    else:
        with emulated_group(world) as run:
            outs = run(rank_fn)
    for rank, out in enumerate(outs):
        if out.shape[0]:
            assert_attention_close(out, expected[rank][0])


def test_wan_entry_follows_token_state(cuda_lib, oracle):
    """wan.sequence_attention with the shared state in token mode (W = 1 here:
    the state is enabled, the group has one rank) equals the Ulysses result."""
    from powershard_b200 import wan
    total, heads = 500, 4
    g = torch.Generator().manual_seed(3)
    q, k, v = (torch.randn(1, total, heads, 128, generator=g).bfloat16().to(DEV) for _ in range(3))
    outs = {}
    for ulysses in (True, False):
        module = type("M", (), {})()
        module.num_heads, module.head_dim = heads, 128
        module._ps_sequence = dict(total=total, enabled=True, ulysses=ulysses, comm_dtype="bf16")
        outs[ulysses] = wan.sequence_attention(module, q, k, v)
        assert module._ps_sequence["kv_collectives"] == 1
    ref = oracle.sdpa_fp32(q.float().cpu(), k.float().cpu(), v.float().cpu())
    assert_attention_close(outs[False], ref)
    assert_attention_close(outs[True], ref)
