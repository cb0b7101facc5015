"""The Ulysses engine over NCCL on several B200s of one node, rank by rank
against the CPU oracle.  Runs when the box exposes
at least `world` GPUs; otherwise reported as skipped (NOT_RUN), never passed.
"""
import json
import os
import socket
from datetime import timedelta
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def nccl_worker(rank, world, port, report, total, heads, exchange):
    import sys
    if str(ROOT) not in sys.path:
        sys.path.insert(0, str(ROOT))
    import __graft_entry__
    __graft_entry__.load_package()
    from oracle import ulysses_oracle as oracle
    from powershard_b200.ulysses import UlyssesAttention
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=dev)
    try:
        g = torch.Generator().manual_seed(3)
        x = [(torch.randn(1, total, heads * 128, generator=g) * 1.4).to(torch.bfloat16) for _ in range(3)]
        wq = torch.rand(heads * 128, generator=g) + 0.5
        wk = torch.rand(heads * 128, generator=g) + 0.5
        freqs = oracle.rope_table_3d((total // 100 + 1, 10, 10), 128)[:, :total]
        a, b = oracle.shard_bounds(total, rank, world)
        token = exchange.startswith("token")
        engine = UlyssesAttention(exchange={"token": "nccl", "token_peer": "peer"}.get(exchange, exchange))
        run = engine.forward_token if token else engine.forward
        state = {}
        outs = []
        for _ in range(2):
            outs.append(run(*(t[0, a:b].to(dev) for t in x), wq.to(dev), wk.to(dev),
                            freqs[0, a:b, 0].to(dev), total=total, heads=heads, state=state))
        engine.check()
        if token:
            expected = oracle.token_sequence_attention(*(t.float() for t in x), wq, wk, freqs, heads,
                                                       world)[rank][0].float()
        else:
            expected = oracle.sequence_attention(x[0], x[1], x[2], wq, wk, freqs, heads, world)[rank][0].float()
        errs = []
        for out in outs:
            err = (out.float().cpu() - expected).abs()
            rel = float(err.mean() / expected.abs().mean()) if expected.numel() else 0.0
            errs.append((float(err.max()) if err.numel() else 0.0, rel))
        ok = all(e <= 2e-2 and r <= 5e-3 for e, r in errs) and state["kv_collectives"] == 2
        ok = ok and state["exchange"] == {"token": "nccl", "token_peer": "peer"}.get(exchange, exchange)
        ok = ok and torch.equal(outs[0], outs[1])
        engine.close()
        Path(f"{report}.{rank}").write_text(json.dumps(dict(ok=ok, errs=errs, rank=rank,
                                                            exchange=state["exchange"])))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("exchange", ["nccl", "peer", "token", "token_peer"])
@pytest.mark.parametrize("world,total,heads", [(2, 1000, 40), (2, 37, 5), (4, 1023, 40), (8, 4099, 40),
                                               (3, 300, 24)])
def test_engine_over_nccl(world, total, heads, exchange, tmp_path, cuda_lib):
    """Both Ulysses exchanges - NCCL all_to_all_single, and the kernels' own
    NVLink peer stores ordered by 4-byte all-reduces (bit-identical results) -
    and token mode (K/V all-gather, local queries)."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"NOT_RUN: needs {world} GPUs, box has {torch.cuda.device_count()}")
    report = tmp_path / "r"
    mp.spawn(nccl_worker, args=(world, _free_port(), str(report), total, heads, exchange), nprocs=world,
             join=True)
    for rank in range(world):
        data = json.loads(Path(f"{report}.{rank}").read_text())
        assert data["ok"], data


def image_worker(rank, world, port, report, prefix, image, heads):
    import sys
    if str(ROOT) not in sys.path:
        sys.path.insert(0, str(ROOT))
    import __graft_entry__
    __graft_entry__.load_package()
    from oracle import ulysses_oracle as oracle
    from powershard_b200.image import SequenceAttention
    from powershard_b200.partition import ImageLayout
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=dev)
    try:
        segments = [(prefix, False), (image, True)]
        g = torch.Generator().manual_seed(4)
        full = [torch.randn(1, prefix + image, heads, 128, generator=g).bfloat16() for _ in range(3)]
        rows = [i for s, e in oracle.image_local_ranges(segments, world, rank) for i in range(s, e)]
        local = [t[:, rows].transpose(1, 2).contiguous().to(dev) for t in full]  # [1, H, n, D]
        stats = {}
        override = SequenceAttention(ImageLayout(segments, world, rank), stats)
        outs = [override(None, *local, heads, skip_reshape=True) for _ in range(2)]
        override.engine.check()
        expected = oracle.image_sequence_attention(*(t.float() for t in full), segments, world)[rank]
        expected = expected.reshape(1, len(rows), heads * 128)
        errs = []
        for out in outs:
            err = (out.float().cpu() - expected).abs()
            errs.append((float(err.max()), float(err.mean() / expected.abs().mean())))
        ok = all(e <= 2e-2 and r <= 5e-3 for e, r in errs) and stats["attention_calls"] == 2
        Path(f"{report}.{rank}").write_text(json.dumps(dict(ok=ok, errs=errs, rank=rank)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,prefix,image,heads", [(2, 512, 4096, 24), (4, 77, 1001, 24), (8, 512, 4096, 24)])
def test_image_override_over_nccl(world, prefix, image, heads, tmp_path, cuda_lib):
    """Flux attention override (configs[4] shape, and a balanced split with
    short middle segments) over NCCL, rank by rank against the oracle."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"NOT_RUN: needs {world} GPUs, box has {torch.cuda.device_count()}")
    report = tmp_path / "r"
    mp.spawn(image_worker, args=(world, _free_port(), str(report), prefix, image, heads), nprocs=world, join=True)
    for rank in range(world):
        data = json.loads(Path(f"{report}.{rank}").read_text())
        assert data["ok"], data


def batch_worker(rank, world, port, report, total, heads, exchange):
    """A CFG batch of 2 rows through forward_batch: one exchange each way for
    the batch (both exchanges), against the oracle row by row."""
    import sys
    if str(ROOT) not in sys.path:
        sys.path.insert(0, str(ROOT))
    import __graft_entry__
    __graft_entry__.load_package()
    from oracle import ulysses_oracle as oracle
    from powershard_b200.ulysses import UlyssesAttention
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=dev)
    try:
        g = torch.Generator().manual_seed(8)
        x = [(torch.randn(2, total, heads * 128, generator=g) * 1.4).to(torch.bfloat16) for _ in range(3)]
        w = torch.rand(heads * 128, generator=g) + 0.5
        freqs = oracle.rope_table_3d((total // 100 + 1, 10, 10), 128)[:, :total]
        a, b = oracle.shard_bounds(total, rank, world)
        engine = UlyssesAttention(exchange=exchange)
        state = {}
        out = engine.forward_batch(*(t[:, a:b].to(dev) for t in x), w.to(dev), w.to(dev), freqs[0, a:b, 0].to(dev),
                                   total=total, heads=heads, state=state)
        engine.check()
        errs = []
        for row in range(2):
            expected = oracle.sequence_attention(x[0][row:row + 1], x[1][row:row + 1], x[2][row:row + 1], w, w,
                                                 freqs, heads, world)[rank][0].float()
            err = (out[row].float().cpu() - expected).abs()
            errs.append((float(err.max()), float(err.mean() / expected.abs().mean())))
        ok = all(e <= 2e-2 and r <= 5e-3 for e, r in errs)
        ok = ok and state["kv_collectives"] == 1 and state["exchange"] == exchange
        ok = ok and state["kv_gathered_bytes"] == world * 3 * 2 * (-(-total // world)) * (-(-heads // world)) * 128 * 2
        engine.close()
        Path(f"{report}.{rank}").write_text(json.dumps(dict(ok=ok, errs=errs, rank=rank)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("exchange", ["nccl", "peer"])
@pytest.mark.parametrize("world,total,heads", [(2, 1000, 40), (4, 1023, 24)])
def test_cfg_batch_over_nccl(world, total, heads, exchange, tmp_path, cuda_lib):
    """Both exchanges with a batch of 2 rows in one call (the reference's
    batched packing, powershard/wan_model.py:356-362)."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"NOT_RUN: needs {world} GPUs, box has {torch.cuda.device_count()}")
    report = tmp_path / "r"
    mp.spawn(batch_worker, args=(world, _free_port(), str(report), total, heads, exchange), nprocs=world, join=True)
    for rank in range(world):
        data = json.loads(Path(f"{report}.{rank}").read_text())
        assert data["ok"], data


def layer_worker(rank, world, port, report, total, heads, fin, exchange):
    """The whole layer (UlyssesAttention.forward_layer: q/k/v GEMM with the
    RMSNorm/RoPE/pack epilogue storing into the exchange, attention, output
    GEMM from the exchange buffer) over a real process group, batch of 2,
    biases on every Linear, against the fp32 layer on this rank's rows."""
    import sys
    for p in (str(ROOT), str(ROOT / "tests")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import __graft_entry__
    __graft_entry__.load_package()
    from oracle import ulysses_oracle as oracle
    from powershard_b200.ulysses import UlyssesAttention
    from test_gpu_layer import assert_layer_close, layer_reference
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=dev)
    try:
        g = torch.Generator().manual_seed(21)
        hid = heads * 128
        x = torch.randn(2, total, fin, generator=g).to(torch.bfloat16).to(dev)
        ws = [(torch.randn(hid, fin, generator=g) * 0.02).to(torch.bfloat16).to(dev) for _ in range(3)]
        ws.append((torch.randn(fin, hid, generator=g) * 0.02).to(torch.bfloat16).to(dev))
        bs = [(torch.randn(n, generator=g) * 0.02).to(dev) for n in (hid, hid, hid, fin)]
        nq = (torch.rand(hid, generator=g) + 0.5).to(dev)
        nk = (torch.rand(hid, generator=g) + 0.5).to(dev)
        table = oracle.rope_table_3d((total // 100 + 1, 10, 10), 128)[0, :total, 0].contiguous().to(dev)
        a, b = oracle.shard_bounds(total, rank, world)
        engine = UlyssesAttention(exchange=exchange)
        state = {}
        out = engine.forward_layer(x[:, a:b].contiguous(), *ws, nq, nk, table[a:b], *bs, total=total, heads=heads,
                                   out_dtype=torch.float32, state=state)
        engine.check()
        ok, msg = True, ""
        if b > a:
            for row in range(2):
                ref = layer_reference(x[row], ws, bs, nq, nk, table, heads)[a:b]
                try:
                    assert_layer_close(out[row], ref, ws[3])
                except AssertionError as exc:
                    ok, msg = False, str(exc)
        ok = ok and state["kv_collectives"] == 1 and state["exchange"] == exchange
        engine.close()
        Path(f"{report}.{rank}").write_text(json.dumps(dict(ok=ok, msg=msg, rank=rank)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,total,heads,fin,exchange", [(2, 1000, 6, 768, "nccl"), (2, 1000, 6, 768, "peer"),
                                                            (4, 1023, 8, 1024, "peer"), (8, 1500, 40, 512, "peer")])
def test_layer_over_nccl(world, total, heads, fin, exchange, tmp_path, cuda_lib):
    """forward_layer with both exchanges on real ranks (the Wan hook's fused
    path, powershard/wan_model.py:421-438 + 441-502)."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"NOT_RUN: needs {world} GPUs, box has {torch.cuda.device_count()}")
    report = tmp_path / "r"
    mp.spawn(layer_worker, args=(world, _free_port(), str(report), total, heads, fin, exchange), nprocs=world,
             join=True)
    for rank in range(world):
        data = json.loads(Path(f"{report}.{rank}").read_text())
        assert data["ok"], data
