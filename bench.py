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
exit 0).
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


def reference_arm(args, world, rank):
    if rank != 0:
        return
    import __graft_entry__  # noqa: F401
    from oracle import ulysses_oracle as oracle
    cores = len(os.sched_getaffinity(0))
    budget = max(1.0, min(10.0, 150.0 / (args.steps + args.warmup)))
    values = []
    last = None
    for step in range(args.warmup + args.steps):
        last = oracle.time_reference_sample(TOTAL, HEADS, DIM, budget_s=budget, threads=cores, seed=step)
        if step >= args.warmup:
            values.append(last["tflops"])
    value = statistics.median(values)
    sample = (f"per step: full pre-pass over {TOTAL} tokens + math_attention (128x512 fp32 tiles) for "
              f"{last['attention_chunks']} of {last['attention_chunks_total']} query chunks (head 0 vs all keys), "
              f"extrapolated to the layer")
    line = dict(metric=METRIC, value=value, unit=UNIT, impl="reference", n_gpus=args.gpus, steps=args.steps,
                warmup=args.warmup, ms_per_step=FLOPS / (value * 1e12) * 1e3, higher_is_better=True,
                scaling="strong", vs_baseline=None, dtype="f32", data="synthetic",
                config=workload_config(args.gpus),
                cpu_baseline=dict(value=value, unit=UNIT, cores=last["threads"], kind="port", sample=sample),
                e2e=dict(value=value, unit=UNIT, h2d_bytes_per_step=0, d2h_bytes_per_step=0))
    print(json.dumps(line), flush=True)


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
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import ulysses_oracle as oracle  # the CPU baseline leg only
        cores = len(os.sched_getaffinity(0))
        res = oracle.time_reference_sample(TOTAL, HEADS, DIM, budget_s=args.cpu_budget, threads=cores)
        cpu = dict(value=res["tflops"], unit=UNIT, cores=res["threads"], kind="port",
                   sample=(f"full pre-pass over {TOTAL} tokens ({res['prepass_s']:.1f} s) + math_attention "
                           f"(128x512 fp32 tiles) for {res['attention_chunks']} of {res['attention_chunks_total']} "
                           f"query chunks of head 0 vs all keys ({res['attention_sample_s']:.1f} s), extrapolated "
                           f"to the layer: {res['seconds_per_layer']:.0f} s/layer"))
    if rank == 0:
        line = dict(
            metric=METRIC, value=flops / (ms * 1e-3) / 1e12, unit=UNIT, n_gpus=world, steps=args.steps,
            warmup=args.warmup, ms_per_step=ms, ms_per_layer=ms, higher_is_better=True, scaling="strong",
            vs_baseline=None, dtype="bf16",
            data="synthetic: x~N(0,1) projected by W~N(0,0.02) (setup), RMSNorm weight 1, RoPE theta 1e4 on 21x30x52",
            config=dict(workload_config(world, total), exchange=exchange),
            roofline=dict(bound="tensor", achieved=achieved, peak=peak, unit="TFLOP/s", frac=achieved / peak,
                          traffic=traffic, kernel="attn_fwd_kernel", attn_ms_per_launch=attn_ms,
                          flops_per_launch=attn_flops, peak_source=peak_src),
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


if __name__ == "__main__":
    main()
