"""The Ulysses exchange logic over real gloo collectives (CPU, no GPU).

``UlyssesAttention`` runs with test-only stand-in kernels (``OracleKernels``)
that fill the same buffers as the CUDA kernels ([W][3][width][h][D] send,
[W][width][h][D] output) from the oracle, so these tests check the host side
of the product path - geometry, buffer reuse, the two all_to_all_single calls,
padding and the state counters - with real multi-process transport, like the
reference's tests/test_sequence_distributed.py.  A rank that leaves between
steps must make the survivor's next exchange raise, not hang.
"""
import json
import os
import time
from datetime import timedelta
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _setup_paths():
    import sys
    if str(ROOT) not in sys.path:
        sys.path.insert(0, str(ROOT))
    import __graft_entry__
    __graft_entry__.load_package()
    from oracle import ulysses_oracle
    return ulysses_oracle


class OracleKernels:
    """Test stand-ins with the buffer contracts of powershard_b200.ops
    (unbatched and batched: a batched call is served row by row)."""

    class DeviceStatus:
        def __init__(self, device):
            self.ptr = None

        def poll(self):
            pass

        def check(self):
            pass

    @classmethod
    def prepass(cls, x_q, x_k, x_v, w_q, w_k, freqs, send, geo, eps=1e-6, norm_rope=True):
        if send.dim() == 6:
            for b in range(send.shape[2]):
                f = freqs[b] if freqs is not None and freqs.dim() == 5 else freqs
                cls.prepass(x_q[b], x_k[b], x_v[b], w_q, w_k, f, send[:, :, b], geo, eps, norm_rope)
            return
        from oracle import ulysses_oracle as oracle
        n, d = geo.n_local, geo.head_dim
        if norm_rope:
            q, k, v = oracle.attention_qkv(x_q[None], x_k[None], x_v[None], w_q, w_k, freqs[None, :, None],
                                           geo.heads, eps)
            q, k, v = q[0], k[0], v[0]
        else:
            q, k, v = (t.reshape(n, geo.heads, d) for t in (x_q, x_k, x_v))
        send.copy_(oracle.pack_qkv(q.to(send.dtype), k.to(send.dtype), v.to(send.dtype), geo.total, geo.rank,
                                   geo.world))

    @classmethod
    def ulysses_attention(cls, recv, out_send, geo, scale, status):
        if recv.dim() == 6:
            for b in range(recv.shape[2]):
                row = out_send[:, b].clone()
                cls.ulysses_attention(recv[:, :, b].contiguous(), row, geo, scale, status)
                out_send[:, b] = row
            return
        from oracle import ulysses_oracle as oracle
        q, k, v = oracle.unpack_qkv(recv, geo.total)
        o = oracle.sdpa_fp32(q[None], k[None], v[None], scale)[0]
        packed = oracle.pack_out(o.to(out_send.dtype), geo.total, geo.world)
        hv = geo.heads_valid
        out_send[..., :hv, :] = packed[..., :hv, :]

    @classmethod
    def unpack(cls, out_recv, out, geo):
        if out_recv.dim() == 5:
            for b in range(out_recv.shape[1]):
                cls.unpack(out_recv[:, b].contiguous(), out[b], geo)
            return
        from oracle import ulysses_oracle as oracle
        out.copy_(oracle.unpack_out(out_recv, geo.total, geo.heads, geo.rank, geo.world).to(out.dtype))

    @staticmethod
    def token_pack(x_q, x_k, x_v, w_q, w_k, freqs, qkv, n_local, heads, head_dim, eps=1e-6, norm_rope=True):
        from oracle import ulysses_oracle as oracle
        if norm_rope:
            q, k, v = oracle.attention_qkv(x_q[None], x_k[None], x_v[None], w_q, w_k, freqs[None, :, None], heads,
                                           eps)
            q, k, v = q[0], k[0], v[0]
        else:
            q, k, v = (t.reshape(n_local, heads, head_dim) for t in (x_q, x_k, x_v))
        qkv.zero_()
        for kind, t in enumerate((q, k, v)):
            qkv[kind, :n_local] = t.to(qkv.dtype)

    @staticmethod
    def token_attention(qkv, kv_all, out, n_local, total, scale, status, workspace=None):
        from oracle import ulysses_oracle as oracle
        world = kv_all.shape[0]
        sizes = [b - a for a, b in (oracle.shard_bounds(total, s, world) for s in range(world))]
        k = torch.cat([kv_all[s, 0, :n] for s, n in enumerate(sizes)])
        v = torch.cat([kv_all[s, 1, :n] for s, n in enumerate(sizes)])
        out.copy_(oracle.sdpa_fp32(qkv[0, :n_local][None], k[None], v[None], scale)[0].to(out.dtype))


class LayoutKernels(OracleKernels):
    """Stand-ins driven by the geometry alone (any token split, including the
    image Layout's balanced one), for the pack-only and joint paths."""

    @classmethod
    def prepass(cls, x_q, x_k, x_v, w_q, w_k, freqs, send, geo, eps=1e-6, norm_rope=True):
        if send.dim() == 6:
            for b in range(send.shape[2]):
                row = send[:, :, b].clone()
                cls.prepass(x_q[b], x_k[b], x_v[b], w_q, w_k, freqs, row, geo, eps, norm_rope)
                send[:, :, b] = row
            return
        assert not norm_rope, "layout stand-in packs pre-normalised inputs only"
        n, h, d = geo.n_local, geo.heads_per_rank, geo.head_dim
        send.zero_()
        for kind, x in enumerate((x_q, x_k, x_v)):
            x = x.reshape(n, geo.heads, d)
            for g in range(geo.heads):
                send[g // h, kind, :n, g % h] = x[:, g]

    @staticmethod
    def ulysses_joint_attention(recv, prefix_qkv, out_send, prefix_out, geo, scale, status):
        from oracle import ulysses_oracle as oracle
        valid = geo.seg_valid()
        hv, plen = geo.heads_valid, prefix_qkv.shape[1]
        q, k, v = (torch.cat([prefix_qkv[kind]] + [recv[s, kind, :valid[s]] for s in range(geo.world)])
                   for kind in range(3))
        o = oracle.sdpa_fp32(q[None, :, :hv], k[None, :, :hv], v[None, :, :hv], scale)[0]
        prefix_out[:, :hv] = o[:plen].to(prefix_out.dtype)
        row = plen
        for s in range(geo.world):
            out_send[s, :valid[s], :hv] = o[row:row + valid[s]].to(out_send.dtype)
            row += valid[s]

    @classmethod
    def unpack(cls, out_recv, out, geo):
        if out_recv.dim() == 5:
            for b in range(out_recv.shape[1]):
                cls.unpack(out_recv[:, b], out[b], geo)
            return
        h = geo.heads_per_rank
        for g in range(geo.heads):
            out[:, g] = out_recv[g // h, :geo.n_local, g % h].to(out.dtype)


def image_layout_worker(rank, world, store, report, prefix, image, heads, batch, skip):
    oracle = _setup_paths()
    from powershard_b200.image import SequenceAttention
    from powershard_b200.partition import ImageLayout
    from powershard_b200.ulysses import UlyssesAttention
    torch.set_num_threads(1)
    dist.init_process_group("gloo", init_method=Path(store).as_uri(), rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))
    try:
        segments = [(prefix, False), (image, True)]
        total = prefix + image
        g = torch.Generator().manual_seed(3)
        q, k, v = (torch.randn(batch, total, heads, 128, generator=g).bfloat16() for _ in range(3))
        lay = ImageLayout(segments, world, rank)
        rows = [i for s, e in oracle.image_local_ranges(segments, world, rank) for i in range(s, e)]
        local = [t[:, rows] for t in (q, k, v)]  # [B, n, H, D]
        if skip:
            local = [t.transpose(1, 2).contiguous() for t in local]  # [B, H, n, D]
        else:
            local = [t.reshape(batch, len(rows), heads * 128) for t in local]
        stats = {}
        override = SequenceAttention(lay, stats, UlyssesAttention(kernels=LayoutKernels))
        called = []
        out = override(lambda *a, **kw: called.append(1), *local, heads, skip_reshape=skip)
        assert not called and stats["attention_calls"] == 1
        expected = oracle.image_sequence_attention(q.float(), k.float(), v.float(), segments, world)[rank]
        assert out.dtype == torch.bfloat16
        torch.testing.assert_close(out.float(), expected.reshape(batch, len(rows), heads * 128), atol=8e-3,
                                   rtol=8e-3)  # one bf16 rounding of the output
        if rank == 0:
            Path(report).write_text(json.dumps(dict(status="PASS", sizes=lay.sizes)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,prefix,image,heads,batch,skip",
                         [(2, 5, 13, 3, 1, True), (3, 4, 13, 5, 2, False), (4, 0, 10, 4, 1, True)])
def test_image_sequence_attention_over_gloo(world, prefix, image, heads, batch, skip, tmp_path, gloo_available):
    """The Flux attention override (text replicated, image split by the
    Layout's balanced sizes) over real gloo collectives: one all-to-all each
    way for image rows, an all-gather over heads for text rows."""
    report = tmp_path / "report.json"
    mp.spawn(image_layout_worker, args=(world, str(tmp_path / "store"), str(report), prefix, image, heads, batch,
                                        skip), nprocs=world, join=True)
    assert json.loads(report.read_text())["status"] == "PASS"


def token_worker(rank, world, store, report, total, heads):
    oracle = _setup_paths()
    from powershard_b200.ulysses import UlyssesAttention
    torch.set_num_threads(1)
    dist.init_process_group("gloo", init_method=Path(store).as_uri(), rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))
    try:
        x, wq, wk, freqs = _inputs(total, heads, oracle)
        a, b = oracle.shard_bounds(total, rank, world)
        engine = UlyssesAttention(kernels=OracleKernels)
        state = {}
        expected = oracle.token_sequence_attention(x[0], x[1], x[2], wq, wk, freqs, heads, world)[rank][0]
        for step in range(2):  # the second step reuses the cached token buffers
            out = engine.forward_token(x[0][0, a:b], x[1][0, a:b], x[2][0, a:b], wq, wk, freqs[0, a:b, 0],
                                       total=total, heads=heads, state=state)
            torch.testing.assert_close(out, expected, atol=1e-5, rtol=1e-5)
        assert state["kv_collectives"] == 2 and "out_collectives" not in state
        assert state["kv_gathered_bytes"] == 2 * 2 * total * heads * 128 * 4
        if rank == 0:
            Path(report).write_text(json.dumps(dict(status="PASS")))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,total,heads", [(2, 41, 5), (3, 41, 3), (4, 9, 2)])
def test_token_mode_over_gloo(world, total, heads, tmp_path, gloo_available):
    """sequence_mode="token": one K/V all-gather per block, local queries, no output exchange."""
    report = tmp_path / "report.json"
    mp.spawn(token_worker, args=(world, str(tmp_path / "store"), str(report), total, heads), nprocs=world,
             join=True)
    assert json.loads(report.read_text())["status"] == "PASS"


def wan_entry_worker(rank, world, store, report, total, heads, ulysses):
    """wan.sequence_attention (the reference's entry, wan_model.py:441-502) on
    each rank: routes by the shared state's mode and keeps its counters."""
    oracle = _setup_paths()
    from powershard_b200 import wan
    from powershard_b200.ulysses import UlyssesAttention
    torch.set_num_threads(1)
    dist.init_process_group("gloo", init_method=Path(store).as_uri(), rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))
    try:
        g = torch.Generator().manual_seed(9)
        q, k, v = (torch.randn(1, total, heads, 128, generator=g) for _ in range(3))
        a, b = oracle.shard_bounds(total, rank, world)
        module = type("SelfAttention", (), {})()
        module.num_heads, module.head_dim = heads, 128
        module._ps_sequence = dict(total=total, enabled=True, ulysses=ulysses, comm_dtype="fp32",
                                   kv_collectives=0, kv_gathered_bytes=0, out_collectives=0, out_exchanged_bytes=0)
        module._ps_b200_engine = UlyssesAttention(kernels=OracleKernels)
        wire = wan.WIRE_DTYPE
        wan.WIRE_DTYPE = torch.float32  # the stand-ins compute in fp32: compare tightly
        try:
            out = wan.sequence_attention(module, q[:, a:b], k[:, a:b], v[:, a:b])
        finally:
            wan.WIRE_DTYPE = wire
        expected = oracle.sdpa_fp32(q, k, v)[:, a:b]
        torch.testing.assert_close(out, expected, atol=1e-5, rtol=1e-5)
        st = module._ps_sequence
        assert st["kv_collectives"] == 1
        assert st["out_collectives"] == (1 if ulysses else 0)
        if rank == 0:
            Path(report).write_text(json.dumps(dict(status="PASS")))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,total,heads,ulysses", [(2, 41, 5, True), (3, 41, 5, False), (2, 9, 3, False)])
def test_wan_entry_over_gloo(world, total, heads, ulysses, tmp_path, gloo_available):
    report = tmp_path / "report.json"
    mp.spawn(wan_entry_worker, args=(world, str(tmp_path / "store"), str(report), total, heads, ulysses),
             nprocs=world, join=True)
    assert json.loads(report.read_text())["status"] == "PASS"


def _inputs(total, heads, oracle):
    g = torch.Generator().manual_seed(7)
    x = [torch.randn(1, total, heads * 128, generator=g) for _ in range(3)]
    wq = torch.rand(heads * 128, generator=g) + 0.5
    wk = torch.rand(heads * 128, generator=g) + 0.5
    freqs = oracle.rope_table_3d((total, 1, 1), 128)
    return x, wq, wk, freqs


def exchange_worker(rank, world, store, report, total, heads):
    oracle = _setup_paths()
    from powershard_b200.ulysses import UlyssesAttention
    torch.set_num_threads(1)
    dist.init_process_group("gloo", init_method=Path(store).as_uri(), rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))
    try:
        x, wq, wk, freqs = _inputs(total, heads, oracle)
        a, b = oracle.shard_bounds(total, rank, world)
        engine = UlyssesAttention(kernels=OracleKernels)
        state = {}
        expected = oracle.sequence_attention(x[0], x[1], x[2], wq, wk, freqs, heads, world,
                                             wire_dtype=torch.float32)[rank][0]
        for step in range(2):  # the second step reuses the cached exchange buffers
            out = engine.forward(x[0][0, a:b], x[1][0, a:b], x[2][0, a:b], wq, wk, freqs[0, a:b, 0],
                                 total=total, heads=heads, state=state)
            torch.testing.assert_close(out, expected, atol=1e-5, rtol=1e-5)
        h = -(-heads // world)
        width = -(-total // world)
        assert state["kv_collectives"] == 2 and state["out_collectives"] == 2
        assert state["padded_heads"] == h * world
        assert state["kv_gathered_bytes"] == 2 * world * 3 * width * h * 128 * 4
        assert state["out_exchanged_bytes"] == 2 * world * width * h * 128 * 4
        if rank == 0:
            Path(report).write_text(json.dumps(dict(status="PASS", world=world, total=total, heads=heads)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,total,heads", [(2, 41, 5), (3, 41, 5), (2, 9, 3), (4, 9, 7)])
def test_ulysses_engine_over_gloo(world, total, heads, tmp_path, gloo_available):
    report = tmp_path / "report.json"
    mp.spawn(exchange_worker, args=(world, str(tmp_path / "store"), str(report), total, heads), nprocs=world,
             join=True)
    assert json.loads(report.read_text())["status"] == "PASS"


def leaving_worker(rank, world, store, report):
    oracle = _setup_paths()
    from powershard_b200.ulysses import UlyssesAttention
    torch.set_num_threads(1)
    dist.init_process_group("gloo", init_method=Path(store).as_uri(), rank=rank, world_size=world,
                            timeout=timedelta(seconds=8))
    total, heads = 17, 4
    x, wq, wk, freqs = _inputs(total, heads, oracle)
    a, b = oracle.shard_bounds(total, rank, world)
    engine = UlyssesAttention(kernels=OracleKernels)
    engine.forward(x[0][0, a:b], x[1][0, a:b], x[2][0, a:b], wq, wk, freqs[0, a:b, 0], total=total, heads=heads)
    dist.barrier()
    if rank == 1:
        os._exit(0)  # leaves between steps: nothing of it is in flight
    start = time.time()
    try:
        engine.forward(x[0][0, a:b], x[1][0, a:b], x[2][0, a:b], wq, wk, freqs[0, a:b, 0], total=total,
                       heads=heads)
        result = "completed"
    except Exception as error:  # the survivor must see an error, not hang
        result = f"{type(error).__name__}: {str(error)[:200]}"
    Path(report).write_text(json.dumps(dict(result=result, seconds=time.time() - start)))
    os._exit(0)  # skip destroy_process_group with a dead peer


def test_rank_leaving_makes_survivor_raise(tmp_path, gloo_available):
    report = tmp_path / "report.json"
    ctx = mp.start_processes(leaving_worker, args=(2, str(tmp_path / "store"), str(report)), nprocs=2,
                             join=False, start_method="spawn")
    deadline = time.time() + 120
    while not ctx.join(timeout=5):
        if time.time() > deadline:
            for p in ctx.processes:
                p.kill()
            pytest.fail("survivor did not finish within 120 s")
    data = json.loads(report.read_text())
    assert data["result"] != "completed", data
    assert data["seconds"] < 60


class H3Kernels(OracleKernels):
    """Stand-ins for the H3 pre-pass: per-head RMSNorm + split-half partial
    RoPE (powershard/attention.py:98-103, :106-181) before the pack."""

    @staticmethod
    def _normed(x_q, x_k, x_v, w_q, w_k, freqs, heads, eps, norm_rope, rope_split_pairs):
        from oracle import ulysses_oracle as oracle
        from powershard_b200 import ops
        assert norm_rope == ops.NORM_PER_HEAD and freqs.shape[-3] == rope_split_pairs
        n = x_q.shape[0]
        table = freqs[None, :, None]
        q, k = (oracle.rope_split_half(oracle.rms_norm_heads(x.reshape(1, n, -1), w, heads, eps)[0], table)
                for x, w in ((x_q, w_q), (x_k, w_k)))
        return q, k, x_v.reshape(n, heads, -1)

    @classmethod
    def prepass(cls, x_q, x_k, x_v, w_q, w_k, freqs, send, geo, eps=1e-6, norm_rope=True, rope_split_pairs=None):
        if send.dim() == 6:
            for b in range(send.shape[2]):
                cls.prepass(x_q[b], x_k[b], x_v[b], w_q, w_k, freqs, send[:, :, b], geo, eps, norm_rope,
                            rope_split_pairs)
            return
        from oracle import ulysses_oracle as oracle
        q, k, v = cls._normed(x_q, x_k, x_v, w_q, w_k, freqs, geo.heads, eps, norm_rope, rope_split_pairs)
        send.copy_(oracle.pack_qkv(q.to(send.dtype), k.to(send.dtype), v.to(send.dtype), geo.total, geo.rank,
                                   geo.world))

    @classmethod
    def token_pack(cls, x_q, x_k, x_v, w_q, w_k, freqs, qkv, n_local, heads, head_dim, eps=1e-6, norm_rope=True,
                   rope_split_pairs=None):
        q, k, v = cls._normed(x_q, x_k, x_v, w_q, w_k, freqs, heads, eps, norm_rope, rope_split_pairs)
        qkv.zero_()
        for kind, t in enumerate((q, k, v)):
            qkv[kind, :n_local] = t.to(qkv.dtype)


def h3_worker(rank, world, store, report, total, heads, ulysses, pairs):
    """h3.attention_forward (replacing powershard/attention.py:106-181) on
    each rank, against per-head norm + split-half RoPE + attention of the
    whole sequence; the module's projection and output are plain matmuls."""
    oracle = _setup_paths()
    from types import SimpleNamespace
    from powershard_b200 import h3
    from powershard_b200.ulysses import UlyssesAttention
    torch.set_num_threads(1)
    dist.init_process_group("gloo", init_method=Path(store).as_uri(), rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))
    try:
        g = torch.Generator().manual_seed(13)
        dim = 64
        x = torch.randn(total, dim, generator=g)
        proj = torch.randn(3 * heads * 128, dim, generator=g) * 0.1
        wq, wk = torch.rand(128, generator=g) + 0.5, torch.rand(128, generator=g) + 0.5
        ang = torch.rand(total, pairs, generator=g, dtype=torch.float64) * 30.0
        c, s = torch.cos(ang), torch.sin(ang)
        table = torch.stack([c, -s, s, c], -1).reshape(1, total, 1, pairs, 2, 2).float()
        q, k, v = (x @ proj.t()).split(heads * 128, dim=-1)
        qn = oracle.rope_split_half(oracle.rms_norm_heads(q[None], wq, heads)[0], table)
        kn = oracle.rope_split_half(oracle.rms_norm_heads(k[None], wk, heads)[0], table)
        expected = oracle.sdpa_fp32(qn[None], kn[None], v.reshape(1, total, heads, 128))[0]
        a, b = oracle.shard_bounds(total, rank, world)
        module = SimpleNamespace(heads=heads, head_dim=128, qkv_proj=lambda t: t @ proj.t(),
                                 q_norm=SimpleNamespace(weight=wq, eps=1e-6),
                                 k_norm=SimpleNamespace(weight=wk, eps=1e-6), out_proj=lambda t: t)
        state = dict(total=total, enabled=True, ulysses=ulysses, comm_dtype="fp32")
        h3.install_attention(module, state=state)
        module._ps_b200_engine = UlyssesAttention(kernels=H3Kernels)
        wire = h3.WIRE_DTYPE
        h3.WIRE_DTYPE = torch.float32  # the stand-ins compute in fp32: compare tightly
        try:
            out = module.forward(x[a:b], table[:, a:b])
        finally:
            h3.WIRE_DTYPE = wire
        assert out.shape == (b - a, heads * 128)
        torch.testing.assert_close(out.reshape(b - a, heads, 128), expected[a:b], atol=1e-5, rtol=1e-5)
        assert state["kv_collectives"] == 1
        if ulysses:
            assert state["out_collectives"] == 1 and state["ulysses_local_heads"] == -(-heads // world)
        else:
            assert "out_collectives" not in state
        if rank == 0:
            Path(report).write_text(json.dumps(dict(status="PASS")))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,total,heads,ulysses,pairs", [(2, 41, 5, True, 32), (3, 40, 4, False, 16),
                                                             (2, 9, 3, False, 64)])
def test_h3_entry_over_gloo(world, total, heads, ulysses, pairs, tmp_path, gloo_available):
    report = tmp_path / "report.json"
    mp.spawn(h3_worker, args=(world, str(tmp_path / "store"), str(report), total, heads, ulysses, pairs),
             nprocs=world, join=True)
    assert json.loads(report.read_text())["status"] == "PASS"


def gather_worker(rank, world, store, report, total, batch):
    """wan.gather_tokens (the final-head gather, powershard/wan_model.py:336-340)
    on each rank against the oracle's gather_rows of every batch row."""
    oracle = _setup_paths()
    from powershard_b200 import wan
    torch.set_num_threads(1)
    dist.init_process_group("gloo", init_method=Path(store).as_uri(), rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))
    try:
        g = torch.Generator().manual_seed(17)
        full = torch.randn(batch, total, 3, 5, generator=g)
        bounds = [oracle.shard_bounds(total, r, world) for r in range(world)]
        a, b = bounds[rank]
        out = wan.gather_tokens(full[:, a:b], total)
        expected = torch.stack([oracle.gather_rows([full[i, s:e] for s, e in bounds], total, world)
                                for i in range(batch)])
        assert torch.equal(out, expected) and torch.equal(out, full) and out.is_contiguous()
        # fp16 wire: values come back in x's dtype, rounded through the wire
        half = wan.gather_tokens(full[:, a:b], total, dtype=torch.float16)
        assert half.dtype == torch.float32 and torch.equal(half, full.half().float())
        # a second call never rewrites the first result
        again = wan.gather_tokens(full[:, a:b] * 2, total)
        assert torch.equal(out, full) and torch.equal(again, full * 2)
        try:
            wan.gather_tokens(torch.zeros(batch, b - a + 1, 3, 5), total)  # raises before any collective
            raise AssertionError("wrong local token count accepted")
        except ValueError:
            pass
        if rank == 0:
            Path(report).write_text(json.dumps(dict(status="PASS")))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,total,batch", [(2, 41, 1), (3, 41, 2), (4, 9, 1)])
def test_head_gather_over_gloo(world, total, batch, tmp_path, gloo_available):
    report = tmp_path / "report.json"
    mp.spawn(gather_worker, args=(world, str(tmp_path / "store"), str(report), total, batch), nprocs=world,
             join=True)
    assert json.loads(report.read_text())["status"] == "PASS"


def batch_worker(rank, world, store, report, golden):
    """wan.self_attention_forward (the hook install_wan_compute sets,
    powershard/wan_model.py:433-438) on a CFG batch of 2 rows over gloo,
    against the reference's recording of the same layer: the whole batch
    crosses in one exchange each way and the counters equal the reference's
    (fp32 wire here, as recorded)."""
    oracle = _setup_paths()
    from powershard_b200 import wan
    from powershard_b200.ulysses import UlyssesAttention
    torch.set_num_threads(1)
    dist.init_process_group("gloo", init_method=Path(store).as_uri(), rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))
    try:
        data = torch.load(golden, weights_only=False)
        case = next(c for c in data["cases"] if c["world"] == world)
        ref = case["ranks"][rank]
        a, b = ref["bounds"]
        heads, hidden = data["heads"], data["x"].shape[-1]
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
        state = dict(total=data["x"].shape[1], enabled=True, ulysses=True, comm_dtype="fp32", kv_collectives=0,
                     kv_gathered_bytes=0, out_collectives=0, out_exchanged_bytes=0)
        module._ps_sequence = state
        engine = UlyssesAttention(kernels=OracleKernels)
        calls = []
        orig_exchange = engine._exchange

        def counted_exchange(recv, send, geo):
            calls.append(tuple(send.shape))
            return orig_exchange(recv, send, geo)
        engine._exchange = counted_exchange
        module._ps_b200_engine = engine
        wire = wan.WIRE_DTYPE
        wan.WIRE_DTYPE = torch.float32  # the recording used the fp32 wire
        try:
            with torch.no_grad():
                out = wan.self_attention_forward(module, data["x"][:, a:b], data["freqs"][:, a:b])
        finally:
            wan.WIRE_DTYPE = wire
        err = (out - ref["out"]).abs()
        assert float(err.max()) <= 2e-2 and float(err.mean() / ref["out"].abs().mean()) <= 5e-3
        # one all_to_all each way, carrying both batch rows
        assert len(calls) == 2 and calls[0][2] == 2 and calls[1][1] == 2, calls
        for key in ("kv_collectives", "kv_gathered_bytes", "out_collectives", "out_exchanged_bytes",
                    "padded_heads"):
            assert state[key] == ref["counters"][key], (key, state[key], ref["counters"][key])
        if rank == 0:
            Path(report).write_text(json.dumps(dict(status="PASS")))
    finally:
        dist.destroy_process_group()


def test_self_attention_forward_cfg_batch_over_gloo(tmp_path, gloo_available):
    report = tmp_path / "report.json"
    golden = ROOT / "tests" / "golden" / "self_attention_forward.pt"
    mp.spawn(batch_worker, args=(2, str(tmp_path / "store"), str(report), str(golden)), nprocs=2, join=True)
    assert json.loads(report.read_text())["status"] == "PASS"
