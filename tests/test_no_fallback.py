"""The product path has no CPU or library fallback: without the built
library, or with tensors that are not on a CUDA device, every entry point
raises before doing any work (CPU only; no GPU needed).

The reference's dispatcher falls back only on UnsupportedAttention raised
before launching (attention_policy.py:135-147); these tests pin which error
each case raises.
"""
from pathlib import Path

import pytest
import torch


def test_missing_library_raises(monkeypatch):
    from powershard_b200 import _lib
    monkeypatch.setattr(_lib, "_LIB", None)
    monkeypatch.setattr(_lib, "LIB_PATH", Path("/nonexistent/libps_b200.so"))
    with pytest.raises(_lib.LibraryMissing):
        _lib.load()


def test_engine_with_cpu_tensors_raises():
    from powershard_b200.contract import UnsupportedAttention
    from powershard_b200.ulysses import UlyssesAttention
    engine = UlyssesAttention()
    x = torch.zeros(8, 2 * 128, dtype=torch.bfloat16)
    w = torch.ones(2 * 128, dtype=torch.bfloat16)
    freqs = torch.zeros(8, 64, 2, 2)
    for run in (engine.forward, engine.forward_token):
        with pytest.raises((UnsupportedAttention, RuntimeError)):
            run(x, x, x, w, w, freqs, total=8, heads=2)


def test_provider_refuses_cpu_and_unsupported_options():
    from powershard_b200 import _lib
    from powershard_b200.contract import AttentionOptions, UnsupportedAttention
    from powershard_b200.provider import B200Provider
    provider = B200Provider.__new__(B200Provider)  # no library load: the checks come first
    provider._status, provider._workspaces = {}, {}
    q = torch.zeros(1, 4, 2, 128, dtype=torch.bfloat16)
    with pytest.raises(UnsupportedAttention):
        provider.check(q, q, q, AttentionOptions(causal=True))
    with pytest.raises(UnsupportedAttention):
        provider.check(q.float(), q.float(), q.float(), AttentionOptions())
    with pytest.raises(UnsupportedAttention):
        provider.check(q[..., :64], q[..., :64], q[..., :64], AttentionOptions())
    with pytest.raises((UnsupportedAttention, RuntimeError)):
        provider.check(q, q, q, AttentionOptions())  # CPU tensors
    assert _lib.UnsupportedAttention is UnsupportedAttention


def test_override_refuses_what_the_kernel_does_not_compute():
    """Masks, keys appended inside the attention and a replicated segment
    after the image go to the fallback or raise, before any launch."""
    from powershard_b200.contract import UnsupportedAttention
    from powershard_b200.image import SequenceAttention
    from powershard_b200.partition import ImageLayout
    lay = ImageLayout([(4, False), (12, True), (3, False)], 1, 0)   # segment after the image
    q = torch.zeros(1, 2, lay.local_len, 128, dtype=torch.bfloat16)
    override = SequenceAttention(lay, {})
    with pytest.raises(UnsupportedAttention):
        override(None, q, q, q, 2, skip_reshape=True)
    seen = []
    fallback = SequenceAttention(lay, {}, fallback=lambda func, *a, **kw: seen.append(1) or "fb")
    assert fallback(None, q, q, q, 2, skip_reshape=True) == "fb" and seen
    with pytest.raises(ValueError):  # wrong local length is a caller error, as in the reference
        override(None, q[:, :, :5], q, q, 2, skip_reshape=True)


def test_geometry_validation():
    from powershard_b200.partition import ImageLayout, UlyssesGeometry, shard_bounds, split_sizes
    with pytest.raises(ValueError):
        UlyssesGeometry(total=10, heads=4, head_dim=128, world=3, rank=0, sizes=(4, 4, 4))  # sums to 12
    with pytest.raises(ValueError):
        UlyssesGeometry(total=10, heads=4, head_dim=128, world=3, rank=0, sizes=(5, 5))     # wrong length
    with pytest.raises(ValueError):
        ImageLayout([(4, False), (8, False)], 2, 0)                                           # no split segment
    with pytest.raises(ValueError):
        shard_bounds(10, 3, 3)
    geo = UlyssesGeometry(total=10, heads=5, head_dim=128, world=3, rank=2, sizes=tuple(split_sizes(10, 3)))
    assert (geo.width, geo.bounds, geo.n_local, geo.heads_per_rank, geo.heads_valid) == (4, (7, 10), 3, 2, 1)
    assert geo.seg_valid() == [4, 3, 3]
    ceil = UlyssesGeometry(total=10, heads=5, head_dim=128, world=3, rank=2)
    assert ceil.seg_valid() == [4, 4, 2] and ceil.bounds == (8, 10)
