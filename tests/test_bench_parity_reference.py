"""bench.py's fp32 restatement of the block (the reference it checks every
run's output rows against) agrees with the pinned CPU oracle: RMSNorm +
RoPE (attention_qkv, powershard/wan_model.py:421-430) followed by fp32
attention, on a small seeded case with several query rows and heads."""
import importlib.util
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parents[1]


def _bench():
    spec = importlib.util.spec_from_file_location("bench_module", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_fp32_block_rows_matches_oracle(oracle):
    bench = _bench()
    from powershard_b200.rope import rope_table_3d
    heads, dim, grid = 3, 128, (2, 5, 7)
    total = grid[0] * grid[1] * grid[2]
    g = torch.Generator().manual_seed(5)
    proj = [(torch.randn(total, heads * dim, generator=g) * 1.3).to(torch.bfloat16) for _ in range(3)]
    w = (torch.rand(heads * dim, generator=g) + 0.5).to(torch.bfloat16)
    table = rope_table_3d(grid, dim)
    rows = [0, 1, 17, 40, total - 1]
    idx = torch.tensor(rows)
    got = bench.fp32_block_rows(proj[0][idx], proj[1], proj[2], w, table[idx], table, heads)
    q, k, v = oracle.attention_qkv(proj[0][None], proj[1][None], proj[2][None], w, w, table[None, :, None], heads)
    ref = oracle.sdpa_fp32(q.float(), k.float(), v.float())[0][idx]
    assert got.shape == (len(rows), heads, dim)
    assert float((got - ref).abs().max()) < 2e-5


def test_sample_rows_cover_edges():
    bench = _bench()
    rows = bench.sample_rows(4095, 64, seed=3)
    assert len(rows) == 64 and rows == sorted(set(rows))
    for r in (0, 4094, 127, 128, 255, 256):
        assert r in rows
    assert bench.sample_rows(5, 64, seed=0) == [0, 1, 2, 3, 4]
