"""Benchmark: Ulysses self-attention block of the Wan2.2-A14B shape on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...      (N > 1, one rank per GPU)

Workload: one self-attention block, L = 32760 tokens
(21x30x52 latent grid), 40 heads x 128, hidden 5120, bf16.  A step is the
whole Ulysses path on every rank: fused q/k RMSNorm + RoPE + pack pre-pass
-> exchange -> tcgen05 attention -> exchange -> unpack.  With --exchange
peer (the default on one node) the pre-pass and the attention epilogue store
across NVLink into the other ranks' buffers and two 4-byte NCCL all-reduces
order the steps; with --exchange nccl two all_to_all_single calls move the
data, as the reference does.  The q/k/v
projections (x ~ N(0,1), W ~ N(0,0.02)) are computed once at setup; they are
the step's inputs.  Inputs (1.0 GB at N=1) exceed the 126 MB L2 and every
step rewrites the exchange buffers, so no extra L2 flush is done.

Rank 0 prints one JSON line: value = 4*L^2*H*D / step time (TFLOP/s, the
whole layer over all N GPUs, max of the per-rank device times); e2e = the
same metric through the public engine with the projections copied from
pinned host memory and the output copied back inside the timed region
(copies on their own streams, overlapping the neighbouring steps' compute);
roofline = the attention kernel's achieved TFLOP/s (CUDA events around each
launch) against the measured bf16 peak; cpu_baseline = the CPU oracle's
restatement of the reference algorithm on a bounded sample (N=1 only).
``--impl reference`` times only that CPU restatement (rank 0; other ranks
exit 0): every step is a bounded, proportional slice of the layer whose
wall time is measured (nothing inside a step is extrapolated).

Outside the timed regions every rank also reports:
  parity  this rank's output against a plain PyTorch fp32 restatement of the
          block (RMSNorm, RoPE, softmax attention) on sampled rows of every
          head, and, at N > 1, the peer-exchange output against the NCCL
          all_to_all exchange (bit-identical); the run exits non-zero when
          parity fails;
  sdpa    torch scaled_dot_product_attention (cuDNN) on the same bf16
          tensors this rank's attention kernel reads, timed the same way;
  comm    (N > 1) bytes each rank sends across NVLink per step and what each
          exchange costs: the peer stores of the fused kernels against the
          same kernels storing locally, and NCCL all_to_all_single;
  layer   the whole layer with its q/k/v/o projections: the fused tcgen05
          GEMMs (forward_layer) against cuBLAS matmuls around the same
          attention path, and each projection GEMM alone.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from datetime import timedelta
from pathlib import Path

import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "Ulysses attn ms/layer & TFLOP/s at 1/2/4/8 B200, Wan-14B 32760-token shape"
UNIT = "TFLOP/s"
TOTAL, HEADS, DIM, GRID = 32760, 40, 128, (21, 30, 52)
HIDDEN = HEADS * DIM
FLOPS = 4.0 * TOTAL * TOTAL * HEADS * DIM
FALLBACK_PEAK_TFLOPS = 1590.0


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=40)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["b200", "reference"], default="b200")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-layer", action="store_true", help="skip the whole-layer (projection GEMMs) report")
    p.add_argument("--cpu-budget", type=float, default=15.0, help="seconds of CPU baseline work")
    p.add_argument("--profile", action="store_true",
                   help="ncu mode: profiler range around the timed steps only; no e2e / CPU baseline")
    p.add_argument("--exchange", choices=["auto", "peer", "nccl"], default="auto",
                   help="how q/k/v and outputs cross ranks: NVLink peer stores or NCCL all_to_all")
    p.add_argument("--seq-len", type=int, default=TOTAL,
                   help="sequence length (default the configs[1] 32760; smaller only for ncu captures)")
    return p.parse_args()


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return float(data["bf16_tflops"]), "measured (MEASURED_PEAKS.json bf16_tflops, burst)"
    return FALLBACK_PEAK_TFLOPS, "fallback 1.59 PFLOP/s"


TRAFFIC_SOURCE = ("ncu dram__bytes_read.sum + dram__bytes_write.sum of one full-size attention launch at W=1 "
                  "(profiles/ncu_traffic.txt); for W > 1 scaled by heads per rank, not measured there")


def traffic_per_launch(world):
    """dram read+write bytes per attention launch from the committed ncu summary."""
    path = ROOT / "profiles" / "ncu_traffic.txt"
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        parts = line.split()
        if len(parts) >= 3 and parts[0] == "attn_fwd" and parts[1] == f"wan14b_w{world}":
            return float(parts[2])
    return None


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples during the timed region."""

    QUERY = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"bench_clocks_{os.getpid()}.csv"

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", str(self.index)], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)

    def stop(self):
        if self.proc is None:
            return dict(sm_mhz=None, sm_max_mhz=None, reasons=["nvidia-smi unavailable"])
        time.sleep(0.15)
        self.proc.terminate()
        self.proc.wait(timeout=10)
        rows = [r.split(", ") for r in self.path.read_text().splitlines() if r.strip()]
        self.path.unlink(missing_ok=True)
        sm = [float(r[2]) for r in rows if len(r) >= 10 and r[2].replace(".", "").isdigit()]
        mx = [float(r[3]) for r in rows if len(r) >= 10 and r[3].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows if len(r) >= 10 for i in range(4) if r[6 + i].strip() == "Active"})
        busy = [s for s in sm if s > 0.5 * (max(sm) if sm else 0)]
        return dict(sm_mhz=statistics.median(busy) if busy else None, sm_max_mhz=max(mx) if mx else None,
                    reasons=reasons, samples=len(sm))


def config0_baseline(cores):
    """configs[0] (Wan2.1-1.3B-shaped layer) over gloo W=2 on the host cores:
    the whole layer of the reference's CPU chain, restated, measured end to
    end per provider, and the committed ratio of that restatement's time to
    the reference's own code measured on the build machine."""
    from oracle import cpu_layer
    res = cpu_layer.time_layer_gloo(world=2, threads=max(1, cores // 2), steps=3, warmup=1)
    pin = ROOT / "oracle" / "config0_timing.json"
    if pin.exists():
        data = json.loads(pin.read_text())
        res["port_vs_reference_code"] = {k: dict(port_over_reference_time=v["port_over_reference_time"],
                                                 max_abs_output_diff=v["max_abs_output_diff"])
                                         for k, v in data["providers"].items()}
        res["port_vs_reference_code"]["measured_on"] = f"{data['cpu_model']}, {data['cores']} cores"
    res["workload"] = "BASELINE configs[0]: x [1, 4096, 1536] fp32, 12x128, q/k/v/o Linear, gloo W=2, whole layer"
    return res


def reference_arm(args, world, rank):
    """The reference's CPU algorithm (oracle restatement, bit-exact to the
    reference's own code on configs[0]) on the host cores.  Each step is a
    bounded slice of the configs[1] layer whose wall time is measured."""
    if rank != 0:
        return
    import __graft_entry__  # noqa: F401
    from oracle import ulysses_oracle as oracle
    cores = len(os.sched_getaffinity(0))
    budget = max(1.0, min(6.0, 150.0 / (args.steps + args.warmup)))
    rates, walls = [], []
    last = None
    t_run = time.perf_counter()
    for step in range(args.warmup + args.steps):
        last = oracle.time_reference_step(TOTAL, HEADS, DIM, budget_s=budget, threads=cores, seed=step)
        if step >= args.warmup:
            rates.append(last["tflops"])
            walls.append(last["wall_s"])
    value = statistics.median(rates)
    sample = (f"per step: math_attention (128x512 fp32 tiles) for {last['chunks']} of {last['chunks_total']} "
              f"(query chunk, head) units against all {TOTAL} keys + the q/k RMSNorm/RoPE/pack pre-pass of "
              f"the same fraction ({last['tokens']} tokens); rate = attention FLOPs executed / step wall time")
    cfg0 = config0_baseline(cores)
    line = dict(metric=METRIC, value=value, unit=UNIT, impl="reference", n_gpus=args.gpus, steps=args.steps,
                warmup=args.warmup, ms_per_step=statistics.median(walls) * 1e3,
                ms_per_layer_extrapolated=FLOPS / (value * 1e12) * 1e3, higher_is_better=True,
                scaling="strong", vs_baseline=None, dtype="f32", data="synthetic",
                hardware=f"host CPU only ({cores} threads), no GPU work",
                config=workload_config(args.gpus),
                cpu_baseline=dict(value=value, unit=UNIT, cores=last["threads"], kind="port", sample=sample,
                                  config0_gloo_w2=cfg0),
                e2e=dict(value=value, unit=UNIT, h2d_bytes_per_step=0, d2h_bytes_per_step=0),
                run_s=time.perf_counter() - t_run)
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------- fp32 check
def fp32_block_rows(q_rows, k_all, v_all, w, freqs_rows, freqs_all, heads, eps=1e-6):
    """Plain PyTorch fp32 restatement of the block for a few query rows:
    RMSNorm over the full width (rounded to the projection dtype, as the
    reference's RMSNorm returns it), interleaved-pair RoPE in fp32, softmax
    attention in fp32 over every key.  q_rows [R, H*D], k_all/v_all [L, H*D]
    projections; returns [R, H, D] fp32."""
    def norm_rope(x, table):
        xf = x.float()
        y = (xf * torch.rsqrt(xf.square().mean(-1, keepdim=True) + eps) * w.float()).to(x.dtype).float()
        y = y.view(x.shape[0], heads, -1, 1, 2)                      # [n, H, D/2, 1, 2]
        rot = table[:, None]                                         # [n, 1, D/2, 2, 2]
        return (rot[..., 0] * y[..., 0] + rot[..., 1] * y[..., 1]).reshape(x.shape[0], heads, -1)
    q = norm_rope(q_rows, freqs_rows)
    k = norm_rope(k_all, freqs_all)
    v = v_all.float().view(v_all.shape[0], heads, -1)
    scale = q.shape[-1] ** -0.5
    s = torch.einsum("rhd,lhd->hrl", q, k) * scale
    p = torch.softmax(s, dim=-1)
    return torch.einsum("hrl,lhd->rhd", p, v)


def sample_rows(n, count, seed):
    """Row indices of a shard: first and last rows, 128-row tile edges and an
    even spread, `count` in all."""
    fixed = {0, 1, 2, n - 3, n - 2, n - 1, 127, 128, 255, 256, n // 2}
    rows = sorted(r for r in fixed if 0 <= r < n)
    g = torch.Generator().manual_seed(seed)
    extra = torch.randperm(n, generator=g).tolist()
    for r in extra:
        if len(rows) >= min(count, n):
            break
        if r not in rows:
            rows.append(r)
    return sorted(rows)


def check_parity(engine_out, proj, norm_w, geo, grid, world, rank, dev, nccl_out=None, rows_per_rank=64):
    """Max-abs / mean-rel error of this rank's output rows (all heads) against
    the fp32 restatement; bit-identity with the NCCL exchange when given."""
    total, heads = geo.total, geo.heads
    from powershard_b200.partition import shard_bounds
    from powershard_b200.rope import rope_table_3d
    freqs_all = rope_table_3d(grid, DIM, device=dev)[:total]
    n = geo.n_local
    width = geo.width
    if world > 1:
        gathered = []
        for t in proj[1:]:
            pad = torch.zeros((width, t.shape[1]), dtype=t.dtype, device=dev)
            pad[:n] = t
            full = torch.empty((world * width, t.shape[1]), dtype=t.dtype, device=dev)
            dist.all_gather_into_tensor(full, pad)
            parts = []
            for r in range(world):
                ra, rb = shard_bounds(total, r, world)
                parts.append(full[r * width: r * width + (rb - ra)])
            gathered.append(torch.cat(parts))
        k_all, v_all = gathered
    else:
        k_all, v_all = proj[1], proj[2]
    a, _ = geo.bounds
    rows = sample_rows(n, rows_per_rank, seed=rank)
    idx = torch.tensor(rows, device=dev)
    prev_tf32 = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        ref = fp32_block_rows(proj[0][idx], k_all, v_all, norm_w, freqs_all[a + idx], freqs_all, heads)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev_tf32
    got = engine_out[idx].float()
    err = (got - ref).abs()
    stats = torch.tensor([float(err.max()), float(err.sum()), float(ref.abs().sum()),
                          0.0 if nccl_out is None or torch.equal(engine_out, nccl_out) else 1.0],
                         device=dev, dtype=torch.float64)
    maxes = stats.clone()
    sums = stats.clone()
    if world > 1:
        dist.all_reduce(maxes, op=dist.ReduceOp.MAX)
        dist.all_reduce(sums, op=dist.ReduceOp.SUM)
    max_abs = float(maxes[0])
    mean_rel = float(sums[1] / sums[2])
    identical = None if nccl_out is None else bool(maxes[3] == 0.0)
    ok = max_abs <= 2e-2 and mean_rel <= 5e-3 and identical is not False
    return dict(ok=ok, max_abs=max_abs, mean_rel=mean_rel, tolerance=dict(max_abs=2e-2, mean_rel=5e-3),
                rows_checked_per_rank=len(rows), heads_checked=heads, ranks=world,
                identical_peer_vs_nccl=identical,
                reference="plain PyTorch fp32 RMSNorm + RoPE + softmax attention over all keys")


def received_qkv(engine, geo, dev):
    """This rank's post-exchange q/k/v [1, h_valid, L, D] (contiguous copies of
    the receive buffer the attention kernel reads)."""
    px = engine._peer(geo, torch.bfloat16, dev, batch=1)
    recv = px.recv if px is not None else engine._workspace(geo, torch.bfloat16, dev, 1)[0]["recv"]
    w, _, _, width, h, d = recv.shape  # [W, 3, B=1, width, h, D]
    hv = geo.heads_valid
    out = []
    for i in range(3):
        t = recv[:, i, 0].reshape(w * width, h, d)[:geo.total, :hv]
        out.append(t.permute(1, 0, 2).unsqueeze(0).contiguous())
    return out


def time_events(fn, reps, warm=2):
    for _ in range(warm):
        fn()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(reps):
        fn()
    e.record()
    e.synchronize()
    return s.elapsed_time(e) / reps


def time_sdpa(q, k, v):
    """torch SDPA (cuDNN backend if it runs, else flash) on this rank's heads."""
    from torch.nn.attention import SDPBackend, sdpa_kernel
    import torch.nn.functional as F
    for backend in (SDPBackend.CUDNN_ATTENTION, SDPBackend.FLASH_ATTENTION):
        try:
            with sdpa_kernel([backend]):
                ms = time_events(lambda: F.scaled_dot_product_attention(q, k, v), reps=5)
            return ms, str(backend).split(".")[-1]
        except RuntimeError:
            continue
    return None, "unavailable"


def measure_comm(engine, proj, norm_w, freqs, geo, dev, ms_step, attn_ms):
    """Per-rank NVLink bytes of one step and the cost of each exchange (max
    over ranks): the fused kernels storing into peers against the same
    kernels storing locally, and NCCL all_to_all_single of the same buffers."""
    from powershard_b200 import ops
    world = geo.world
    esize = 2
    block_qkv = 3 * geo.width * geo.heads_per_rank * DIM * esize
    block_out = geo.width * geo.heads_per_rank * DIM * esize
    qkv_bytes, out_bytes = (world - 1) * block_qkv, (world - 1) * block_out
    local_send = torch.empty(geo.send_shape(), dtype=torch.bfloat16, device=dev)
    local_stage = torch.empty((geo.width, geo.padded_heads, DIM), dtype=torch.bfloat16, device=dev)
    status = ops.DeviceStatus(dev)
    ws = ops.attention_workspace(dev)
    scale = DIM ** -0.5
    res = {}

    def sync_all():
        torch.cuda.synchronize(dev)
        dist.barrier(device_ids=[dev.index])

    px = engine._peer(geo, torch.bfloat16, dev, batch=1)  # the buffers the timed steps used
    if px is not None:
        local_blocks = [local_stage.data_ptr() + r * geo.heads_per_rank * DIM * esize for r in range(world)]
        xb = [t[None] for t in proj]
        attn = dict(workspace=ws, batch=1, out_batch_stride=px.out_batch_stride)
        runs = dict(
            prepass_to=lambda: ops.prepass_to(*xb, norm_w, norm_w, freqs, px.dst_blocks, geo, torch.bfloat16, batch=1),
            prepass_local=lambda: ops.prepass(*proj, norm_w, norm_w, freqs, local_send, geo),
            attn_to=lambda: ops.ulysses_attention_to(px.recv, px.out_blocks, px.out_row_stride, torch.bfloat16, geo,
                                                     scale, status, **attn),
            attn_local=lambda: ops.ulysses_attention_to(px.recv, local_blocks, px.out_row_stride, torch.bfloat16,
                                                        geo, scale, status, **attn))
        # Peer-storing and local-storing launches alternate (same clocks and
        # power state for both); each figure is the median of its launches.
        samples = {k: [] for k in runs}
        for rep in range(4):
            for name in ("prepass_to", "prepass_local", "attn_to", "attn_local"):
                sync_all()
                samples[name].append(time_events(runs[name], reps=1, warm=1 if rep == 0 else 0))
        sync_all()
        res["peer"] = {f"{k}_ms": statistics.median(v) for k, v in samples.items()}
    recv = torch.empty_like(local_send)
    out_send = torch.empty(geo.out_shape(), dtype=torch.bfloat16, device=dev)
    out_recv = torch.empty_like(out_send)
    sync_all()
    t_a2a_qkv = time_events(lambda: dist.all_to_all_single(recv, local_send), reps=5)
    sync_all()
    t_a2a_out = time_events(lambda: dist.all_to_all_single(out_recv, out_send), reps=5)
    sync_all()
    res["nccl"] = dict(qkv_a2a_ms=t_a2a_qkv, out_a2a_ms=t_a2a_out)
    status.check()
    # max over ranks of every time
    keys = [(k, kk) for k in res for kk in res[k]]
    vals = torch.tensor([res[k][kk] for k, kk in keys], device=dev, dtype=torch.float64)
    dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    for (k, kk), v in zip(keys, vals.tolist()):
        res[k][kk] = v
    gbs = lambda nbytes, ms: nbytes / (ms * 1e-3) / 1e9 if ms and ms > 0 else None  # noqa: E731
    if "peer" in res:
        pr = res["peer"]
        pr["qkv_added_ms"] = pr["prepass_to_ms"] - pr["prepass_local_ms"]
        pr["out_added_ms"] = pr["attn_to_ms"] - pr["attn_local_ms"]
        pr["qkv_gbs_over_kernel"] = gbs(qkv_bytes, pr["prepass_to_ms"])
        pr["out_gbs_over_kernel"] = gbs(out_bytes, pr["attn_to_ms"])
    nc = res["nccl"]
    nc["qkv_gbs"] = gbs(qkv_bytes, nc["qkv_a2a_ms"])
    nc["out_gbs"] = gbs(out_bytes, nc["out_a2a_ms"])
    res.update(qkv_bytes_per_rank=qkv_bytes, out_bytes_per_rank=out_bytes,
               link_gbs_nominal=900.0, link_gbs_measured_peer_copy=770.0,
               step_minus_attention_ms=ms_step - attn_ms,
               note="bytes each rank sends to the other ranks per step (bf16 wire); GB/s = bytes / time of "
                    "the step that moves them; added_ms = peer-storing kernel minus the same kernel storing "
                    "locally")
    return res


def measure_layer(engine, geo, freqs, dev, world, reps=3, rounds=3):
    """The whole self-attention layer (powershard/wan_model.py:421-438) of the
    configs[1] shape, outside the headline timing: x [1, n, 5120] bf16 and
    random bf16 q/k/v/o weights.  fused = UlyssesAttention.forward_layer (the
    q/k/v GEMM with RMSNorm + RoPE + pack in its epilogue, exchange,
    attention, output GEMM reading the exchange buffer); cublas = torch
    matmuls for the four projections around the same attention path
    (engine.forward).  Per-launch times of the projection GEMMs come from
    CUDA events around each launch; every time is the max over ranks."""
    from powershard_b200 import ops
    n, total = geo.n_local, geo.total
    g = torch.Generator(device=dev).manual_seed(2000 + geo.rank)
    x = torch.randn(1, n, HIDDEN, device=dev, dtype=torch.bfloat16, generator=g)
    ws = [(torch.randn(HIDDEN, HIDDEN, device=dev, generator=g) * 0.02).to(torch.bfloat16) for _ in range(4)]
    norm = torch.ones(HIDDEN, device=dev, dtype=torch.float32)
    kw = dict(total=total, heads=HEADS, local=world == 1)

    def sync_all():
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier(device_ids=[dev.index])

    def fused():
        return engine.forward_layer(x, *ws, norm, norm, freqs, **kw)

    def cublas():
        q, k, v = (x[0] @ w.t() for w in ws[:3])
        o = engine.forward(q, k, v, norm, norm, freqs, **kw)
        return o.view(n, HIDDEN) @ ws[3].t()

    events = {"qkv_projection": [], "out_projection": []}
    orig = {name: getattr(ops, name) for name in events}

    def timed(name):
        def run(*a_, **k_):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            orig[name](*a_, **k_)
            e.record()
            events[name].append((s, e))
        return run

    # The two paths alternate (same clocks and power state for both: the SM
    # clock drifts under the power cap); each figure is the median of its
    # rounds.
    samples = {"cublas": [], "fused": [], "gemm_qkv": [], "gemm_o": []}
    for rnd in range(rounds):
        sync_all()
        samples["cublas"].append(time_events(cublas, reps, warm=2 if rnd == 0 else 1))
        samples["gemm_qkv"].append(time_events(lambda: [x[0] @ w.t() for w in ws[:3]], reps, warm=1))
        samples["gemm_o"].append(time_events(lambda: x[0] @ ws[3].t(), reps, warm=1))
        sync_all()
        for name in events:
            setattr(ops, name, timed(name))
        try:
            samples["fused"].append(time_events(fused, reps, warm=2 if rnd == 0 else 1))
        finally:
            for name, fn in orig.items():
                setattr(ops, name, fn)
    t_cublas, t_fused = statistics.median(samples["cublas"]), statistics.median(samples["fused"])
    t_gemm_qkv, t_gemm_o = statistics.median(samples["gemm_qkv"]), statistics.median(samples["gemm_o"])
    sync_all()
    engine.check()
    per = {k: statistics.median(s.elapsed_time(e) for s, e in v) for k, v in events.items()}
    vals = torch.tensor([t_fused, t_cublas, per["qkv_projection"], per["out_projection"], t_gemm_qkv, t_gemm_o],
                        device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    t_fused, t_cublas, t_qkv, t_o, t_gemm_qkv, t_gemm_o = vals.tolist()
    e2e_wan = measure_e2e_wan(x, ws, norm, freqs, geo, dev, world, reps)
    attn_flops = 4.0 * total * total * HEADS * DIM
    proj_flops = 2.0 * total * HIDDEN * HIDDEN * 4          # the whole layer's four projections
    del x, ws
    tf = lambda flops, ms: flops / (ms * 1e-3) / 1e12  # noqa: E731
    return dict(
        fused_ms=t_fused, cublas_ms=t_cublas, fused_over_cublas_time=t_fused / t_cublas,
        layer_tflops_fused=tf(attn_flops + proj_flops, t_fused),
        layer_tflops_cublas=tf(attn_flops + proj_flops, t_cublas),
        qkv_gemm_ms=t_qkv, qkv_gemm_tflops=tf(6.0 * n * HIDDEN * HIDDEN, t_qkv),
        qkv_cublas_ms=t_gemm_qkv, qkv_cublas_tflops=tf(6.0 * n * HIDDEN * HIDDEN, t_gemm_qkv),
        out_gemm_ms=t_o, out_gemm_tflops=tf(2.0 * n * HIDDEN * HIDDEN, t_o),
        out_cublas_ms=t_gemm_o, out_cublas_tflops=tf(2.0 * n * HIDDEN * HIDDEN, t_gemm_o),
        rounds=rounds, reps_per_round=reps, e2e_wan=e2e_wan,
        what="whole layer, x [1, n_local, 5120] bf16 -> [1, n_local, 5120]: fused = forward_layer (qkv GEMM with "
             "RMSNorm/RoPE/pack epilogue, exchange, attention, o GEMM from the exchange buffer); cublas = torch "
             "matmuls + engine.forward (pre-pass, exchange, attention, unpack); *_gemm = the fused GEMM kernels "
             "alone (events around each launch), *_cublas = torch matmuls of the same shapes (q/k/v: three)")


def measure_e2e_wan(x, ws, norm, freqs, geo, dev, world, reps):
    """The layer end to end through the entry a PowerShard worker installs:
    wan.self_attention_forward on a module with bf16 q/k/v/o Linear layers
    and RMSNorm q/k (the shape install_wan_compute routes), x copied from
    pinned host memory and the output copied back every step, in order on
    one stream.  Max over ranks."""
    from powershard_b200 import wan
    n = geo.n_local
    module = torch.nn.Module()
    for name, w in zip("qkvo", ws):
        lin = torch.nn.Linear(HIDDEN, HIDDEN, bias=False, device=dev, dtype=torch.bfloat16)
        lin.weight.data.copy_(w)
        setattr(module, name, lin)
    module.norm_q = torch.nn.RMSNorm(HIDDEN, eps=1e-6, device=dev)
    module.norm_k = torch.nn.RMSNorm(HIDDEN, eps=1e-6, device=dev)
    module.norm_q.weight.data.copy_(norm)
    module.norm_k.weight.data.copy_(norm)
    module.num_heads, module.head_dim = HEADS, DIM
    module._ps_sequence = dict(total=geo.total, enabled=world > 1, ulysses=True, comm_dtype="bf16")
    table = freqs[None, :, None]
    host_x = x.cpu().pin_memory()
    host_out = torch.empty_like(host_x).pin_memory()
    dev_x = torch.empty_like(x)

    def step():
        dev_x.copy_(host_x, non_blocking=True)
        with torch.no_grad():
            out = wan.self_attention_forward(module, dev_x, table)
        host_out.copy_(out, non_blocking=True)

    for _ in range(2):
        step()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier(device_ids=[dev.index])
    ms = time_events(step, reps, warm=0)
    module._ps_b200_engine.check()
    fused = getattr(module, "_ps_b200_fused_cache", None) is not None
    val = torch.tensor([ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(val, op=dist.ReduceOp.MAX)
        module._ps_b200_engine.close()
    ms = float(val[0])
    nbytes = n * HIDDEN * 2
    return dict(ms_per_layer=ms, fused_layer=fused, h2d_bytes_per_step=nbytes, d2h_bytes_per_step=nbytes,
                attn_tflops=4.0 * geo.total * geo.total * HEADS * DIM / (ms * 1e-3) / 1e12,
                what="wan.self_attention_forward (the hook worker.install_network installs), bf16 Linear layers, "
                     "pinned-host x in and layer output out each step, serial on one stream")


def workload_config(world, total=TOTAL):
    name = "Wan2.2-A14B self-attention block (configs[1])" if total == TOTAL else f"Wan-14B block, L={total}"
    return dict(workload=name, seq_len=total, heads=HEADS,
                head_dim=DIM, hidden=HIDDEN, latent_grid="21x30x52", global_batch=1, world=world,
                parallelism=f"ulysses{world}",
                l2="inputs 1.0 GB > 126 MB L2 and each step rewrites the exchange buffers (no flush)",
                excluded="q/k/v/o projection GEMMs (cuBLAS, computed once at setup / outside the path)")


def main():
    args = parse()
    world, rank, local = dist_env()
    if args.impl == "reference":
        reference_arm(args, world, rank)
        return
    import __graft_entry__
    __graft_entry__.build()
    from powershard_b200 import ops
    from powershard_b200.partition import UlyssesGeometry
    from powershard_b200.rope import rope_table_3d
    from powershard_b200.ulysses import UlyssesAttention

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=dev)
    total = args.seq_len
    flops = 4.0 * total * total * HEADS * DIM
    geo = UlyssesGeometry(total=total, heads=HEADS, head_dim=DIM, world=world, rank=rank)
    a, b = geo.bounds
    n = geo.n_local

    # ---- inputs: projections of x ~ N(0,1) by W ~ N(0, 0.02), computed once.
    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    x = torch.randn(n, HIDDEN, device=dev, dtype=torch.bfloat16, generator=g)
    proj = []
    for _ in range(3):
        w = (torch.randn(HIDDEN, HIDDEN, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        proj.append(x @ w.t())
        del w
    del x
    norm_w = torch.ones(HIDDEN, device=dev, dtype=torch.bfloat16)
    grid = GRID if total == TOTAL else (math.ceil(total / (GRID[1] * GRID[2])), GRID[1], GRID[2])
    freqs = rope_table_3d(grid, DIM, device=dev)[a:b].contiguous()
    engine = UlyssesAttention(exchange=args.exchange)

    # Attention-kernel timing: events around each launch on the launch stream.
    attn_events = []
    orig_attention = {name: getattr(ops, name) for name in ("ulysses_attention", "ulysses_attention_to")}

    def timed(name):
        def run(*a_, **k_):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            orig_attention[name](*a_, **k_)
            e.record()
            attn_events.append((s, e))
        return run

    def step(inputs):
        return engine.forward(*inputs, norm_w, norm_w, freqs, total=total, heads=HEADS)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize(dev)

    state = {}
    engine.forward(*proj, norm_w, norm_w, freqs, total=total, heads=HEADS, state=state)
    for _ in range(args.warmup):
        step(proj)
    engine.check()
    exchange = state.get("exchange", "local")
    clocks = ClockSampler(local)
    clocks.start()
    for name in orig_attention:
        setattr(ops, name, timed(name))
    barrier()
    if args.profile:
        torch.cuda.profiler.start()
    from powershard_b200 import _lib
    launches0 = _lib.load().ps_b200_kernel_launches()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(args.steps):
        step(proj)
    t1.record()
    launches = _lib.load().ps_b200_kernel_launches() - launches0
    barrier()
    if args.profile:
        torch.cuda.profiler.stop()
    for name, fn in orig_attention.items():
        setattr(ops, name, fn)
    clock = clocks.stop()
    engine.check()
    ms = t0.elapsed_time(t1) / args.steps
    attn_ms = statistics.mean(s.elapsed_time(e) for s, e in attn_events)

    if args.profile:
        if rank == 0:
            print(json.dumps(dict(profile=True, seq_len=total, n_gpus=world, ms_per_step=ms,
                                  attn_ms_per_launch=attn_ms)), flush=True)
        if world > 1:
            engine.close()
            dist.destroy_process_group()
        return

    # ---- e2e: public engine, host (pinned) inputs and output every step,
    # pipelined as a serving loop runs it: each step's H2D copy runs on its own
    # stream into one of two device input sets, the engine call waits for it,
    # and the D2H copy of the output runs on a third stream, so copies of
    # neighbouring steps overlap compute.  Every copy is inside the timed region.
    host_in = [t.cpu().pin_memory() for t in proj]
    host_out = [torch.empty((n, HEADS, DIM), dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    dev_in = [[torch.empty_like(t) for t in proj] for _ in range(2)]
    compute = torch.cuda.current_stream(dev)
    h2d_stream, d2h_stream = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    freed = [None, None]  # event: the compute stream is done with dev_in[slot]
    e2e_steps = max(4, args.steps // 2)

    def e2e_step(k):
        slot = k % 2
        with torch.cuda.stream(h2d_stream):
            if freed[slot] is not None:
                h2d_stream.wait_event(freed[slot])
            for d_, h_ in zip(dev_in[slot], host_in):
                d_.copy_(h_, non_blocking=True)
            loaded = torch.cuda.Event()
            loaded.record(h2d_stream)
        compute.wait_event(loaded)
        out = step(dev_in[slot])
        done = torch.cuda.Event()
        done.record(compute)
        freed[slot] = done
        with torch.cuda.stream(d2h_stream):
            d2h_stream.wait_event(done)
            host_out[slot].copy_(out, non_blocking=True)
            out.record_stream(d2h_stream)

    for k in range(2):
        e2e_step(k)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(h2d_stream)
    for k in range(e2e_steps):
        e2e_step(k)
    e1.record(d2h_stream)
    barrier()
    e2e_ms = e0.elapsed_time(e1) / e2e_steps
    h2d = sum(t.numel() * t.element_size() for t in host_in)
    d2h = host_out[0].numel() * host_out[0].element_size()

    if world > 1:
        vals = torch.tensor([ms, e2e_ms, attn_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
        ms, e2e_ms, attn_ms = vals.tolist()
    peak, peak_src = peaks()
    attn_flops = 4.0 * total * total * geo.heads_valid * DIM
    achieved = attn_flops / (attn_ms * 1e-3) / 1e12
    traffic = traffic_per_launch(world)

    # ---- outside the timed regions: parity, SDPA on the same tensors, comm.
    out_main = step(proj)
    nccl_out = None
    if world > 1 and exchange == "peer":
        nccl_engine = UlyssesAttention(exchange="nccl")
        nccl_out = nccl_engine.forward(*proj, norm_w, norm_w, freqs, total=total, heads=HEADS)
        nccl_engine.check()
    engine.check()
    parity = check_parity(out_main, proj, norm_w, geo, grid, world, rank, dev, nccl_out=nccl_out)
    del nccl_out
    q_s, k_s, v_s = received_qkv(engine, geo, dev)
    sdpa_ms, sdpa_backend = time_sdpa(q_s, k_s, v_s)
    del q_s, k_s, v_s
    sdpa_vals = torch.tensor([sdpa_ms if sdpa_ms is not None else -1.0], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(sdpa_vals, op=dist.ReduceOp.MAX)
    sdpa_ms = float(sdpa_vals[0]) if float(sdpa_vals[0]) > 0 else None
    sdpa = dict(backend=sdpa_backend, ms_per_launch=sdpa_ms,
                tflops=attn_flops / (sdpa_ms * 1e-3) / 1e12 if sdpa_ms else None,
                kernel_over_sdpa_time=attn_ms / sdpa_ms if sdpa_ms else None,
                what="torch scaled_dot_product_attention on this rank's post-exchange q/k/v [1, h, L, 128] bf16, "
                     "CUDA events, max over ranks")
    comm = measure_comm(engine, proj, norm_w, freqs, geo, dev, ms, attn_ms) if world > 1 else None
    del proj
    layer = None
    if not args.no_layer:
        # Outside the timed region and not part of the metric: a failure here
        # (argument checks fail alike on every rank, before any collective) is
        # reported in the line instead of ending the run.
        try:
            layer = measure_layer(engine, geo, freqs, dev, world)
        except Exception as exc:  # noqa: BLE001 - reported in the line, never fatal to the metric
            layer = dict(error=f"{type(exc).__name__}: {str(exc)[:300]}")

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import ulysses_oracle as oracle  # the CPU baseline leg only
        cores = len(os.sched_getaffinity(0))
        res = oracle.time_reference_step(TOTAL, HEADS, DIM, budget_s=args.cpu_budget, threads=cores)
        cpu = dict(value=res["tflops"], unit=UNIT, cores=res["threads"], kind="port",
                   sample=(f"math_attention (128x512 fp32 tiles) for {res['chunks']} of {res['chunks_total']} "
                           f"(query chunk, head) units against all {TOTAL} keys + the pre-pass of the same "
                           f"fraction ({res['tokens']} tokens), {res['wall_s']:.1f} s measured; the layer at "
                           f"this rate: {FLOPS / (res['tflops'] * 1e12):.0f} s"),
                   config0_gloo_w2=config0_baseline(cores))
    if rank == 0:
        line = dict(
            metric=METRIC, value=flops / (ms * 1e-3) / 1e12, unit=UNIT, n_gpus=world, steps=args.steps,
            warmup=args.warmup, ms_per_step=ms, ms_per_layer=ms, higher_is_better=True, scaling="strong",
            vs_baseline=None, dtype="bf16",
            data="synthetic: x~N(0,1) projected by W~N(0,0.02) (setup), RMSNorm weight 1, RoPE theta 1e4 on 21x30x52",
            config=workload_config(world, total), exchange=exchange,
            roofline=dict(bound="tensor", achieved=achieved, peak=peak, unit="TFLOP/s", frac=achieved / peak,
                          traffic=traffic, traffic_source=TRAFFIC_SOURCE, kernel="attn_fwd_kernel",
                          attn_ms_per_launch=attn_ms, flops_per_launch=attn_flops, peak_source=peak_src),
            parity=parity, sdpa=sdpa, comm=comm, layer=layer,
            cpu_baseline=cpu,
            e2e=dict(value=flops / (e2e_ms * 1e-3) / 1e12, unit=UNIT, ms_per_step=e2e_ms,
                     h2d_bytes_per_step=h2d, d2h_bytes_per_step=d2h,
                     pipelining="H2D and D2H on their own streams, two device input sets"),
            clocks=clock, gpu_launches=int(launches))
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local])
        engine.close()
        dist.destroy_process_group()
    if not parity["ok"]:
        sys.exit(3)


if __name__ == "__main__":
    main()
