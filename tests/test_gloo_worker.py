"""Worker integration (powershard/wan_backend.py:413-496) over real gloo ranks.

``tests/golden/wan_backend_call.pt`` holds what the reference's own
``WanBackend.call`` returned for a forward of a two-block stand-in network
whose blocks run the reference's ``self_attention_forward`` (Ulysses and
token mode, W=2, fp32 wire, math provider): each rank's output, the shared
sequence state after the forward and ``metrics["sequence_communication"]``.

Here the same network is built from torch modules, routed through the b200
path with ``worker.install_network`` (the counterpart of install_wan_compute's
self-attention branch), and run by two gloo ranks with the same forward
(the sequence handling of wan_forward: counters reset, blocks, head gather).
The kernels are the test stand-ins of test_gloo_ulysses (the CUDA kernels
need a B200; tests/test_gpu_worker.py runs them).  The b200 state must carry
the reference's counters, so ``worker.sequence_communication`` - the metrics
block WanBackend.call builds from that state - equals the recorded one.
"""
import json
from datetime import timedelta
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden" / "wan_backend_call.pt"
COUNTERS = ("kv_collectives", "kv_gathered_bytes", "out_collectives", "out_exchanged_bytes", "scale_collectives",
            "head_gathers", "effective_comm_dtype")


def build_network(data, state):
    """The recorded two-block network as torch modules, routed through b200."""
    from powershard_b200 import worker

    class Block(torch.nn.Module):
        def __init__(self, weights, norms):
            super().__init__()
            hidden = weights[0].shape[0]
            for name, w in zip("qkvo", weights):
                lin = torch.nn.Linear(hidden, hidden)
                lin.weight.data.copy_(w)
                lin.bias.data.zero_()
                setattr(self, name, lin)
            self.norm_q = torch.nn.RMSNorm(hidden, eps=data["eps"])
            self.norm_k = torch.nn.RMSNorm(hidden, eps=data["eps"])
            self.norm_q.weight.data.copy_(norms[0])
            self.norm_k.weight.data.copy_(norms[1])
            self.num_heads, self.head_dim = data["heads"], hidden // data["heads"]

    net = torch.nn.Module()
    net.blocks = torch.nn.ModuleList([Block(w, n) for w, n in zip(data["weights"], data["norms"])])
    routed = worker.install_network(net, state)
    return net, routed


def forward(net, x, freqs, state, total):
    """The sequence handling of wan_forward (powershard/wan_model.py:1004-1011,
    :1073-1075) around the blocks: counters reset, residual blocks on this
    rank's tokens, final-head gather."""
    from powershard_b200 import wan
    from powershard_b200.partition import shard_bounds
    world, rank = dist.get_world_size(), dist.get_rank()
    state.update(total=total, enabled=world > 1, kv_collectives=0, kv_gathered_bytes=0, out_collectives=0,
                 out_exchanged_bytes=0, scale_collectives=0, head_gathers=0)
    a, b = shard_bounds(total, rank, world)
    local = x[:, a:b]
    for blk in net.blocks:
        local = local + blk(local, freqs[:, a:b])
    out = wan.gather_tokens(local, total)
    state["head_gathers"] += 1
    return out


def worker_rank(rank, world, store, report, mode):
    import sys
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "tests"))
    import __graft_entry__
    __graft_entry__.load_package()
    from powershard_b200 import wan, worker
    from powershard_b200.ulysses import UlyssesAttention
    from test_gloo_ulysses import OracleKernels
    torch.set_num_threads(1)
    dist.init_process_group("gloo", init_method=Path(store).as_uri(), rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))
    try:
        data = torch.load(GOLDEN, weights_only=False)
        case = next(c for c in data["cases"] if c["mode"] == mode)
        ref = case["ranks"][rank]
        state = dict(total=0, enabled=False, ulysses=mode == "ulysses", comm_dtype="fp32", mode=mode)
        net, routed = build_network(data, state)
        assert routed == ["blocks.0", "blocks.1"], routed
        engine = UlyssesAttention(kernels=OracleKernels)   # one engine per rank, shared by the blocks
        for blk in net.blocks:
            blk._ps_b200_engine = engine
            assert blk._ps_sequence is state
        wire = wan.WIRE_DTYPE
        wan.WIRE_DTYPE = torch.float32                       # the recording used the fp32 wire
        try:
            with torch.no_grad():
                x = data["x"]
                out = forward(net, x, data["freqs"], state, x.shape[1])
        finally:
            wan.WIRE_DTYPE = wire
        delta, ref_delta = out - x, ref["out"] - x           # the blocks' contribution
        err = (delta - ref_delta).abs()
        assert float(err.max()) <= 2e-2 and float(err.mean() / ref_delta.abs().mean()) <= 5e-3
        for key in COUNTERS:
            assert state[key] == ref["state"][key], (key, state[key], ref["state"][key])
        if mode == "ulysses":
            assert state["padded_heads"] == ref["state"]["padded_heads"]
        assert worker.sequence_communication(state) == ref["sequence_communication"]
        if rank == 0:
            Path(report).write_text(json.dumps(dict(status="PASS", metrics=ref["sequence_communication"])))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["ulysses", "token"])
def test_wan_backend_forward_metrics_over_gloo(mode, tmp_path, gloo_available):
    report = tmp_path / "report.json"
    mp.spawn(worker_rank, args=(2, str(tmp_path / "store"), str(report), mode), nprocs=2, join=True)
    assert json.loads(report.read_text())["status"] == "PASS"


def test_install_network_skips_non_self_attention():
    """Cross-attention and plain layers keep their forward; only modules with
    the self-attention shape (q/k/v/o, norm_q/norm_k, heads) are routed."""
    from powershard_b200 import worker

    class SelfAttn(torch.nn.Module):
        def __init__(self):
            super().__init__()
            for name in "qkvo":
                setattr(self, name, torch.nn.Linear(8, 8))
            self.norm_q, self.norm_k = torch.nn.RMSNorm(8), torch.nn.RMSNorm(8)
            self.num_heads, self.head_dim = 1, 8

    class WanT2VCrossAttention(SelfAttn):
        pass

    net = torch.nn.Module()
    net.a = SelfAttn()
    net.c = WanT2VCrossAttention()
    net.ffn = torch.nn.Linear(8, 8)
    routed = worker.install_network(net)
    assert routed == ["a"]
    assert net.a._ps_sequence is net._ps_sequence
    assert "forward" in net.a.__dict__ and "forward" not in net.c.__dict__
    assert worker.sequence_communication(net._ps_sequence) is None
