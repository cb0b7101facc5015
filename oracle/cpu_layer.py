"""Whole Wan self-attention layer on CPU ranks over gloo (TEST INFRASTRUCTURE).

The timed CPU baseline of BASELINE configs[0]: a Wan2.1-1.3B-shaped layer
(x [1, 4096, 1536] fp32, 12 heads x 128, 16x16x16 token grid) run by
``world`` spawned processes that exchange tensors with real
``all_to_all_single`` calls over gloo.  Each rank runs the reference's chain
for its token shard, restated in plain PyTorch:

  q/k/v Linear (operations.Linear, fp32)          powershard/wan_model.py:425-429
  attention_qkv: RMSNorm(q), RMSNorm(k) + rope_apply  wan_model.py:421-430
  ulysses_to_sequence (pad, pack, all_to_all)     wan_model.py:343-364
  run_attention: power-of-two scales, fp16 cast,  wan_model.py:385-418
      provider "math" (attention_contract.py:85-125) or "sdpa" (:128-145)
  ulysses_to_heads (pack, all_to_all, unpack)     wan_model.py:367-381
  o Linear                                        wan_model.py:438

Only ``bench.py`` (its CPU-baseline leg and ``--impl reference`` arm) and
``oracle/time_config0.py`` run it; nothing in the product imports it.
"""
from __future__ import annotations

import math
import os
import statistics
import time
from datetime import timedelta

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from . import ulysses_oracle as ref

CONFIG0 = dict(grid=(16, 16, 16), hidden=1536, heads=12, head_dim=128, eps=1e-6, seed=0)


def layer_inputs(cfg=CONFIG0):
    """Seeded configs[0] inputs: x ~ N(0,1) [1, L, hidden], q/k/v/o weights
    ~ N(0, 0.02) with zero bias, RMSNorm weights 1, the 3-D RoPE table."""
    g = torch.Generator().manual_seed(cfg["seed"])
    total = math.prod(cfg["grid"])
    hidden = cfg["hidden"]
    x = torch.randn(1, total, hidden, generator=g)
    weights = [torch.randn(hidden, hidden, generator=g) * 0.02 for _ in range(4)]
    freqs = ref.rope_table_3d(cfg["grid"], cfg["head_dim"])
    return x, weights, freqs


def _all_to_all(send):
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send)
    return recv


def layer_forward(x_local, weights, freqs_local, total, heads, provider, eps=1e-6):
    """One rank's layer: [1, n, hidden] fp32 -> [1, n, hidden] fp32 over the
    initialised process group (fp32 wire, the reference's default)."""
    world, rank = dist.get_world_size(), dist.get_rank()
    wq, wk, wv, wo = weights
    hidden = x_local.shape[-1]
    dim = hidden // heads
    ones = torch.ones(hidden)
    q_lin, k_lin, v_lin = x_local @ wq.t(), x_local @ wk.t(), x_local @ wv.t()
    q, k, v = ref.attention_qkv(q_lin, k_lin, v_lin, ones, ones, freqs_local, heads, eps)
    send = ref.pack_qkv(q[0], k[0], v[0], total, rank, world)
    recv = _all_to_all(send)
    qg, kg, vg = ref.unpack_qkv(recv, total)
    # run_attention (wan_model.py:398-418) with static scales 1: q/k cast to
    # fp16, v divided by its power-of-two scale before the cast.
    sv = ref._power2_scale(vg.abs().amax() / 16384.0) if vg.numel() else torch.ones(())
    q16, k16, v16 = qg[None].half(), kg[None].half(), (vg[None] / sv).half()
    if provider == "math":
        o = ref.math_attention(q16, k16, v16)
    else:
        o = torch.nn.functional.scaled_dot_product_attention(
            q16.transpose(1, 2).float(), k16.transpose(1, 2).float(), v16.transpose(1, 2).float()
        ).transpose(1, 2).to(torch.float16)
    o = o[0].float() * sv
    back = _all_to_all(ref.pack_out(o, total, world).contiguous())
    out = ref.unpack_out(back, total, heads, rank, world)
    n = x_local.shape[1]
    return out.reshape(1, n, heads * dim) @ wo.t()


def _worker(rank, world, port, threads, steps, warmup, providers, queue):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.set_num_threads(threads)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=300))
    try:
        cfg = CONFIG0
        x, weights, freqs = layer_inputs(cfg)
        total = x.shape[1]
        a, b = ref.shard_bounds(total, rank, world)
        result = {}
        with torch.no_grad():
            for provider in providers:
                times = []
                for step in range(warmup + steps):
                    dist.barrier()
                    t0 = time.perf_counter()
                    layer_forward(x[:, a:b], weights, freqs[:, a:b], total, cfg["heads"], provider, cfg["eps"])
                    dist.barrier()
                    if step >= warmup:
                        times.append(time.perf_counter() - t0)
                result[provider] = times
        queue.put((rank, result))
    finally:
        dist.destroy_process_group()


def time_layer_gloo(world=2, threads=None, steps=5, warmup=1, providers=("math", "sdpa"), port=None):
    """Median wall seconds per layer (barrier to barrier) of configs[0] over
    gloo with ``world`` spawned ranks of ``threads`` threads each (default:
    the host cores split evenly), per provider."""
    cores = len(os.sched_getaffinity(0))
    threads = threads or max(1, cores // world)
    if port is None:
        import socket
        with socket.socket() as sock:  # a free local port, away from any torchrun rendezvous
            sock.bind(("127.0.0.1", 0))
            port = sock.getsockname()[1]
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, threads, steps, warmup, providers, queue))
             for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            rank, res = queue.get(timeout=900)
            results[rank] = res
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    per_provider = {}
    total = math.prod(CONFIG0["grid"])
    flops = 4.0 * total * total * CONFIG0["heads"] * CONFIG0["head_dim"]
    for provider in providers:
        step_s = [max(results[r][provider][i] for r in range(world)) for i in range(steps)]
        med = statistics.median(step_s)
        per_provider[provider] = dict(ms_per_layer=med * 1e3, attn_tflops=flops / med / 1e12,
                                      steps_s=[round(t, 4) for t in step_s])
    return dict(world=world, threads_per_rank=threads, cores=cores, steps=steps, warmup=warmup,
                providers=per_provider)
