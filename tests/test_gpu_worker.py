"""Worker integration on the CUDA path (needs a B200): the two-block network
of tests/golden/wan_backend_call.pt routed through the b200 kernels with
worker.install_network, against the reference's own WanBackend.call
recording - at W=1 (sequence state off) and with two ranks emulated on one
GPU (Ulysses and token mode, the bf16 wire: the recorded fp32-wire byte
counters halve)."""
import pytest
import torch

from test_gloo_worker import COUNTERS, GOLDEN, build_network, forward

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def _delta_close(out, x, ref):
    delta, ref_delta = (out - x).float(), (ref - x).float()
    err = (delta - ref_delta).abs()
    assert float(err.max()) <= 2e-2 and float(err.mean() / ref_delta.abs().mean()) <= 5e-3


def test_network_world1_matches_reference_call(cuda_lib):
    import torch.distributed as dist
    data = torch.load(GOLDEN, weights_only=False)
    state = dict(total=0, enabled=False, ulysses=True, comm_dtype="bf16")
    net, routed = build_network(data, state)
    net = net.to(DEV)
    assert routed == ["blocks.0", "blocks.1"]
    x = data["x"].to(DEV)
    assert not dist.is_initialized()
    with torch.no_grad():
        local = x
        for blk in net.blocks:
            local = local + blk(local, data["freqs"].to(DEV))
    for blk in net.blocks:
        blk._ps_b200_engine.check()
    _delta_close(local.cpu(), data["x"], data["cases"][0]["ranks"][0]["out"])


@pytest.mark.parametrize("mode", ["ulysses", "token"])
def test_network_emulated_two_ranks_metrics(cuda_lib, mode):
    from emulated_dist import emulated_group
    from powershard_b200 import worker
    data = torch.load(GOLDEN, weights_only=False)
    case = next(c for c in data["cases"] if c["mode"] == mode)

    def rank_fn(rank):
        state = dict(total=0, enabled=False, ulysses=mode == "ulysses", comm_dtype="bf16", mode=mode)
        net, _ = build_network(data, state)
        net = net.to(DEV)
        x = data["x"].to(DEV)
        with torch.no_grad():
            out = forward(net, x, data["freqs"].to(DEV), state, x.shape[1])
        for blk in net.blocks:
            blk._ps_b200_engine.check()
        return out.cpu(), state

    with emulated_group(2) as run:
        results = run(rank_fn)
    for rank, (out, state) in enumerate(results):
        ref = case["ranks"][rank]
        _delta_close(out, data["x"], ref["out"])
        for key in COUNTERS:
            want = ref["state"][key]
            if key.endswith("_bytes"):
                want = want // 2            # bf16 wire against the recorded fp32 wire
            if key == "effective_comm_dtype":
                want = "bfloat16"
            assert state[key] == want, (key, state[key], want)
        comm = worker.sequence_communication(state)
        ref_comm = dict(ref["sequence_communication"], communication_dtype="bfloat16",
                        exchanged_bytes=ref["sequence_communication"]["exchanged_bytes"] // 2)
        assert comm == ref_comm
