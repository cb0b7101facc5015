"""CUDA graph capture of the b200 calls (needs a B200): a captured call
replays to the eager result, follows new input data written into the
captured tensors, and the kernels still report through the status word."""
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def test_graphed_engine_block_matches_eager(cuda_lib, oracle):
    from powershard_b200.graphs import GraphedCall
    from powershard_b200.rope import rope_table_3d
    from powershard_b200.ulysses import UlyssesAttention
    total, heads = 1000, 4
    g = torch.Generator(device=DEV).manual_seed(4)
    x = [torch.randn(total, heads * 128, device=DEV, generator=g).bfloat16() for _ in range(3)]
    w = torch.ones(heads * 128, dtype=torch.bfloat16, device=DEV)
    f = rope_table_3d((10, 10, 10), 128, device=DEV)
    engine = UlyssesAttention()
    kw = dict(total=total, heads=heads, local=True)
    eager = engine.forward(*x, w, w, f, **kw).clone()
    graphed = GraphedCall(engine.forward, *x, w, w, f, **kw)
    out = graphed()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    x[0].copy_(torch.randn(total, heads * 128, device=DEV, generator=g).bfloat16())   # new queries
    expected = engine.forward(*x, w, w, f, **kw).clone()
    out = graphed()
    engine.check()
    assert torch.equal(out, expected) and not torch.equal(out, eager)


def test_graphed_flux_override_and_provider(cuda_lib, oracle):
    from powershard_b200.contract import AttentionOptions
    from powershard_b200.graphs import GraphedCall
    from powershard_b200.image import SequenceAttention
    from powershard_b200.partition import ImageLayout
    from powershard_b200.provider import B200Provider
    g = torch.Generator(device=DEV).manual_seed(5)
    lay = ImageLayout([(77, False), (1000, True)], 1, 0)
    q, k, v = (torch.randn(1, 6, lay.local_len, 128, device=DEV, generator=g).bfloat16() for _ in range(3))
    override = SequenceAttention(lay, {})
    eager = override(None, q, k, v, 6, skip_reshape=True).clone()
    graphed = GraphedCall(override, None, q, k, v, 6, skip_reshape=True)
    assert torch.equal(graphed(), eager)
    provider = B200Provider()
    qb = q.transpose(1, 2)
    eager_p = provider(qb, qb, qb, AttentionOptions()).clone()
    graphed_p = GraphedCall(provider, qb, qb, qb, AttentionOptions())
    out = graphed_p()
    torch.cuda.synchronize()
    assert torch.equal(out, eager_p)
