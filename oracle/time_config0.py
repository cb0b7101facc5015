"""Time the reference's own CPU layer against its restatement.

Run where a ComfyUI-PowerShard source tree is available, naming it:

    POWERSHARD_REFERENCE=<path to the ComfyUI-PowerShard tree> python -m oracle.time_config0

Two gloo ranks (spawned processes, host cores split evenly) run the
Wan2.1-1.3B-shaped layer of BASELINE configs[0] twice per provider
("math", the reference default, and "sdpa"):

* the reference itself: ``wan_model.self_attention_forward`` (attention_qkv
  + sequence_attention + o, powershard/wan_model.py:421-502) on a module
  built from ``operations.Linear`` / ``operations.RMSNorm`` with an
  ``AttentionDispatcher`` of that provider, Ulysses mode, fp32 wire;
* the restatement ``oracle.cpu_layer.layer_forward`` that ``bench.py``
  times on the GPU box's host (the reference tree does not travel there).

It writes ``oracle/config0_timing.json``: median wall ms per layer of each
(implementation, provider), the port/reference time ratio, the largest
output difference between the two, the cores and the CPU model.  The
ratio is what ties the GPU box's port timing to the reference's own code.
"""
from __future__ import annotations

import json
import math
import os
import platform
import statistics
import sys
import time
from datetime import timedelta
from pathlib import Path
from types import SimpleNamespace

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent


def _cpu_model():
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return platform.processor() or "unknown"


def _worker(rank, world, port, threads, steps, warmup, ref_root, queue):
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ref_root))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.set_num_threads(threads)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=600))
    try:
        from oracle import cpu_layer, ulysses_oracle as port
        from powershard import wan_model
        from powershard.attention_policy import AttentionDispatcher
        from powershard.config import DistributedConfig
        from powershard.operations import Linear, RMSNorm

        cfg = cpu_layer.CONFIG0
        x, weights, freqs = cpu_layer.layer_inputs(cfg)
        total, hidden, heads = x.shape[1], cfg["hidden"], cfg["heads"]
        a, b = port.shard_bounds(total, rank, world)
        result = {}
        for provider in ("math", "sdpa"):
            dcfg = DistributedConfig(attention_backend=provider, sequence_mode="ulysses")
            lin = []
            for w in weights:
                layer = Linear(hidden, hidden, bias=True)
                layer.weight.data.copy_(w)
                layer.bias.data.zero_()
                lin.append(layer)
            norm_q, norm_k = RMSNorm(hidden, eps=cfg["eps"]), RMSNorm(hidden, eps=cfg["eps"])
            norm_q.weight.data.fill_(1.0)
            norm_k.weight.data.fill_(1.0)
            state = wan_model.new_sequence_state(dcfg)
            state.update(total=total, enabled=True, kv_collectives=0, kv_gathered_bytes=0, out_collectives=0,
                         out_exchanged_bytes=0, padded_heads=0, scale_collectives=0)
            mod = SimpleNamespace(num_heads=heads, head_dim=cfg["head_dim"], norm_q=norm_q, norm_k=norm_k,
                                  q=lin[0], k=lin[1], v=lin[2], o=lin[3], _ps_qk_scales=(1., 1., 1.),
                                  _ps_sequence=state, _ps_attention=AttentionDispatcher(dcfg),
                                  _ps_group="wan_self", _ps_safe=False)
            runs = dict(
                reference=lambda: wan_model.self_attention_forward(mod, x[:, a:b], freqs[:, a:b]),
                port=lambda: cpu_layer.layer_forward(x[:, a:b], weights, freqs[:, a:b], total, heads, provider,
                                                     cfg["eps"]))
            outs = {}
            for name, fn in runs.items():
                times = []
                with torch.no_grad():
                    for step in range(warmup + steps):
                        dist.barrier()
                        t0 = time.perf_counter()
                        out = fn()
                        dist.barrier()
                        if step >= warmup:
                            times.append(time.perf_counter() - t0)
                outs[name] = out
                result[(name, provider)] = times
            result[("diff", provider)] = float((outs["reference"] - outs["port"]).abs().max())
        queue.put((rank, result))
    finally:
        dist.destroy_process_group()


def main(steps=5, warmup=1, world=2):
    ref_root = os.environ.get("POWERSHARD_REFERENCE")
    if not ref_root or not (Path(ref_root) / "powershard").is_dir():
        raise SystemExit("set POWERSHARD_REFERENCE to a ComfyUI-PowerShard source tree")
    cores = len(os.sched_getaffinity(0))
    threads = max(1, cores // world)
    port = 29600 + os.getpid() % 1000
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, threads, steps, warmup, ref_root, queue))
             for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, res = queue.get(timeout=3600)
        results[rank] = res
    for p in procs:
        p.join()
    from oracle import cpu_layer
    total = math.prod(cpu_layer.CONFIG0["grid"])
    flops = 4.0 * total * total * cpu_layer.CONFIG0["heads"] * cpu_layer.CONFIG0["head_dim"]
    out = dict(config="BASELINE configs[0]: Wan2.1-1.3B-shaped layer, x [1, 4096, 1536] fp32, 12x128, "
                      "16x16x16 grid, Ulysses over gloo",
               world=world, threads_per_rank=threads, cores=cores, cpu_model=_cpu_model(),
               torch=torch.__version__, steps=steps, warmup=warmup, providers={})
    for provider in ("math", "sdpa"):
        entry = {}
        for name in ("reference", "port"):
            step_s = [max(results[r][(name, provider)][i] for r in range(world)) for i in range(steps)]
            med = statistics.median(step_s)
            entry[name] = dict(ms_per_layer=round(med * 1e3, 2), attn_tflops=flops / med / 1e12)
        entry["port_over_reference_time"] = entry["port"]["ms_per_layer"] / entry["reference"]["ms_per_layer"]
        entry["max_abs_output_diff"] = max(results[r][("diff", provider)] for r in range(world))
        out["providers"][provider] = entry
    path = HERE / "config0_timing.json"
    path.write_text(json.dumps(out, indent=1) + "\n")
    print(json.dumps(out, indent=1))


if __name__ == "__main__":
    main()
