"""Generate the golden fixtures that pin the CPU oracle to the reference.

Run once where a ComfyUI-PowerShard source tree is available, naming it:

    POWERSHARD_REFERENCE=<path to the ComfyUI-PowerShard tree> python tests/golden/make_golden.py

It imports the reference package from that tree (torch only, no ComfyUI),
runs the reference's own hot-path functions on seeded inputs and saves
inputs + outputs with torch.save next to this script:

* ``attention_qkv.pt``  - operations.RMSNorm + wan_model.rope_apply through
  wan_model.attention_qkv (fp32 and bf16 projections).
* ``rope_split_half.pt`` - attention.rope_split_half (H3 partial RoPE).
* ``ulysses_exchange.pt`` - attention.ulysses_heads_to_sequence ->
  math_attention -> ulysses_sequence_to_heads for W in {3,4,5,6}, heads 7 and
  56, 2W+1 tokens, D=8, V*1e6 (the geometry of the reference's own
  tests/test_sequence_distributed.py), plus wan_model.ulysses_to_sequence /
  ulysses_to_heads at D=128.
* ``math_attention.pt`` - attention_contract.math_attention cases.
* ``sequence_attention.pt`` - wan_model.sequence_attention (Ulysses, math
  provider, fp32 wire) for W in {1,2,3} on a 40-token, 5-head, D=128 layer;
  ``sequence_attention_token.pt`` the same in token mode (K/V all-gather).
* ``self_attention_forward.pt`` - wan_model.self_attention_forward (q/k/v/o
  operations.Linear + RMSNorm, attention_qkv, sequence_attention, o) on a
  CFG batch of 2 rows, W=1 (sequence state off, math provider) and Ulysses
  W=2 (math provider, fp32 wire), with the state counters of each rank.
* ``wan_backend_call.pt`` - wan_backend.WanBackend.call (the worker's forward
  command) over a two-block stand-in network whose blocks run the
  reference's self_attention_forward with residuals and whose forward keeps
  the sequence state as wan_forward does (counters reset, head gather), at
  W=2 in Ulysses and token mode (math provider, fp32 wire): the output of
  each rank, the state after the forward and metrics["sequence_communication"].
* ``image_sequence_attention.pt`` - image_parallel.SequenceAttention (the
  Flux/Qwen attention override: local queries, all-gathered keys/values)
  over image_layout.Layout for uneven image segments, W in {2,3,5}, with a
  dense fp32 stand-in for ComfyUI's optimized_attention as `func`.

Collectives are emulated in-process with one thread per rank (the same
technique as the reference's test_ulysses_tensor_permutation_reference).
"""
from __future__ import annotations

import os
import sys
import threading
from concurrent.futures import ThreadPoolExecutor
from contextlib import contextmanager
from pathlib import Path
from types import SimpleNamespace

import torch
import torch.distributed as dist

HERE = Path(__file__).resolve().parent
REF = Path(os.environ["POWERSHARD_REFERENCE"]) if "POWERSHARD_REFERENCE" in os.environ else None


@contextmanager
def emulated_collectives(world):
    """Patch torch.distributed with a thread-per-rank in-process transport."""
    local = threading.local()
    barrier = threading.Barrier(world, timeout=60)
    slots = [None] * world
    saved = {n: getattr(dist, n) for n in ("get_world_size", "get_rank", "all_to_all_single",
                                           "all_gather_into_tensor", "all_reduce", "get_backend")}

    def all_to_all(output, input, group=None):
        slots[local.rank] = input.clone()
        barrier.wait()
        output.copy_(torch.stack([slots[r][local.rank] for r in range(world)]))
        barrier.wait()

    def all_gather(output, input, group=None):
        slots[local.rank] = input.clone()
        barrier.wait()
        output.copy_(torch.cat(slots))
        barrier.wait()

    def all_reduce(value, op=None, group=None):
        slots[local.rank] = value.clone()
        barrier.wait()
        value.copy_(torch.stack(slots).amax(0))
        barrier.wait()

    dist.get_world_size = lambda group=None: world
    dist.get_rank = lambda group=None: local.rank
    dist.all_to_all_single = all_to_all
    dist.all_gather_into_tensor = all_gather
    dist.all_reduce = all_reduce
    dist.get_backend = lambda group=None: "nccl"  # selects all_gather_into_tensor in image_parallel

    def run(fn):
        def worker(rank):
            local.rank = rank
            try:
                return fn(rank)
            except BaseException:
                barrier.abort()
                raise
        with ThreadPoolExecutor(max_workers=world) as ex:
            return list(ex.map(worker, range(world)))
    try:
        yield run
    finally:
        for n, f in saved.items():
            setattr(dist, n, f)


def rope_table(n, pairs, seed):
    g = torch.Generator().manual_seed(seed)
    ang = torch.rand(n, pairs, generator=g, dtype=torch.float64) * 40.0
    c, s = torch.cos(ang), torch.sin(ang)
    return torch.stack([c, -s, s, c], -1).reshape(1, n, 1, pairs, 2, 2).float()


def main():
    if REF is None or not (REF / "powershard").is_dir():
        raise SystemExit("set POWERSHARD_REFERENCE to a ComfyUI-PowerShard source tree")
    sys.path.insert(0, str(REF))
    torch.set_num_threads(4)
    from powershard import wan_model, attention
    from powershard.attention_contract import AttentionOptions, math_attention
    from powershard.attention_policy import AttentionDispatcher
    from powershard.config import DistributedConfig, shard_bounds
    from powershard.operations import RMSNorm

    # ---------------------------------------------------------- attention_qkv
    cases = []
    for dtype in (torch.float32, torch.bfloat16):
        g = torch.Generator().manual_seed(11)
        n, heads, dim = 37, 3, 128
        q_lin, k_lin, v_lin = (torch.randn(1, n, heads * dim, generator=g).to(dtype) * 1.7 for _ in range(3))
        wq = (torch.rand(heads * dim, generator=g) + 0.5).to(dtype)
        wk = (torch.rand(heads * dim, generator=g) + 0.5).to(dtype)
        freqs = rope_table(n, dim // 2, 5)
        norm_q, norm_k = RMSNorm(heads * dim, eps=1e-6, dtype=dtype), RMSNorm(heads * dim, eps=1e-6, dtype=dtype)
        norm_q.weight.data.copy_(wq)
        norm_k.weight.data.copy_(wk)
        mod = SimpleNamespace(num_heads=heads, head_dim=dim, norm_q=norm_q, norm_k=norm_k,
                              q=lambda x, t=q_lin: t, k=lambda x, t=k_lin: t, v=lambda x, t=v_lin: t)
        with torch.no_grad():
            q, k, v = wan_model.attention_qkv(mod, torch.zeros(1, n, heads * dim), freqs)
        cases.append(dict(dtype=str(dtype), heads=heads, eps=1e-6, q_lin=q_lin, k_lin=k_lin, v_lin=v_lin,
                          wq=wq, wk=wk, freqs=freqs, q=q, k=k, v=v))
    torch.save(cases, HERE / "attention_qkv.pt")

    # H3 partial RoPE (split half) on bf16 / fp32 rows.
    rcases = []
    for dtype, pairs in ((torch.float32, 32), (torch.bfloat16, 64), (torch.bfloat16, 16)):
        g = torch.Generator().manual_seed(41 + pairs)
        x = (torch.randn(29, 3, 128, generator=g) * 2.0).to(dtype)
        table = rope_table(29, pairs, 7 + pairs)
        rcases.append(dict(x=x, table=table, out=attention.rope_split_half(x, table)))
    torch.save(rcases, HERE / "rope_split_half.pt")

    # ------------------------------------------------------ Ulysses exchange
    exchange = []
    for world in (3, 4, 5, 6):
        for heads in (7, 56):
            total, dim = 2 * world + 1, 8
            gen = torch.Generator().manual_seed(991)
            q, k = (torch.randn(total, heads, dim, generator=gen) for _ in range(2))
            v = torch.randn(total, heads, dim, generator=gen) * 1e6

            def rank_fn(rank):
                a, b = shard_bounds(total, rank, world)
                (qg, kg, vg), padded, nbytes = attention.ulysses_heads_to_sequence(
                    (q[a:b], k[a:b], v[a:b]), total, heads)
                got = math_attention(qg[None], kg[None], vg[None], AttentionOptions(), 3, 5)[0]
                local = attention.ulysses_sequence_to_heads(got, total, heads)
                return dict(qg=qg, kg=kg, vg=vg, padded=padded, nbytes=nbytes, attn=got, out=local)
            with emulated_collectives(world) as run:
                per_rank = run(rank_fn)
            exchange.append(dict(layout="LHD", world=world, heads=heads, total=total, dim=dim,
                                 q=q, k=k, v=v, ranks=per_rank))
    # Batch-first Wan helpers at D=128, uneven heads and tokens.
    for world in (2, 3):
        total, heads, dim = 2 * world + 3, 5, 128
        gen = torch.Generator().manual_seed(17)
        q, k, v = (torch.randn(1, total, heads, dim, generator=gen) for _ in range(3))

        def rank_fn(rank):
            a, b = shard_bounds(total, rank, world)
            (qg, kg, vg), padded, nbytes = wan_model.ulysses_to_sequence(
                (q[:, a:b], k[:, a:b], v[:, a:b]), total, heads)
            back, nbytes_out = wan_model.ulysses_to_heads(qg, total, heads)
            return dict(qg=qg, kg=kg, vg=vg, padded=padded, nbytes=nbytes, back=back, nbytes_out=nbytes_out)
        with emulated_collectives(world) as run:
            per_rank = run(rank_fn)
        exchange.append(dict(layout="BLHD", world=world, heads=heads, total=total, dim=dim,
                             q=q, k=k, v=v, ranks=per_rank))
    torch.save(exchange, HERE / "ulysses_exchange.pt")

    # --------------------------------------------------------- math_attention
    mcases = []
    g = torch.Generator().manual_seed(9)
    for (b, lq, lk, h, scale, qc, kc) in ((2, 5, 7, 4, .13, 2, 3), (2, 5, 7, 4, .37, 128, 512),
                                          (1, 300, 300, 2, None, 128, 512), (1, 129, 513, 1, .09, 128, 512)):
        q = torch.randn(b, lq, h, 128, generator=g)
        k = torch.randn(b, lk, h, 128, generator=g)
        v = torch.randn(b, lk, h, 128, generator=g)
        out = math_attention(q, k, v, AttentionOptions(softmax_scale=scale), qc, kc)
        mcases.append(dict(q=q, k=k, v=v, scale=scale, query_chunk=qc, key_chunk=kc, out=out))
    torch.save(mcases, HERE / "math_attention.pt")

    # ------------------------------------------------------ sequence_attention
    scases = []
    n_total, heads, dim = 40, 5, 128
    g = torch.Generator().manual_seed(23)
    q_lin, k_lin, v_lin = (torch.randn(1, n_total, heads * dim, generator=g) for _ in range(3))
    wq = torch.rand(heads * dim, generator=g) + 0.5
    wk = torch.rand(heads * dim, generator=g) + 0.5
    freqs = rope_table(n_total, dim // 2, 3)
    tcases = []
    for mode, world in [("ulysses", w) for w in (1, 2, 3)] + [("token", w) for w in (1, 2, 3)]:
        cfg = DistributedConfig(attention_backend="math", sequence_mode=mode)

        def rank_fn(rank):
            a, b = shard_bounds(n_total, rank, world)
            norm_q, norm_k = RMSNorm(heads * dim, eps=1e-6), RMSNorm(heads * dim, eps=1e-6)
            norm_q.weight.data.copy_(wq)
            norm_k.weight.data.copy_(wk)
            state = wan_model.new_sequence_state(cfg)
            state.update(total=n_total, enabled=True, kv_collectives=0, kv_gathered_bytes=0, out_collectives=0,
                         out_exchanged_bytes=0, padded_heads=0, scale_collectives=0)
            mod = SimpleNamespace(num_heads=heads, head_dim=dim, norm_q=norm_q, norm_k=norm_k,
                                  q=lambda x: q_lin[:, a:b], k=lambda x: k_lin[:, a:b], v=lambda x: v_lin[:, a:b],
                                  _ps_qk_scales=(1., 1., 1.), _ps_sequence=state,
                                  _ps_attention=AttentionDispatcher(cfg), _ps_group="wan_self", _ps_safe=False)
            with torch.no_grad():
                q, k, v = wan_model.attention_qkv(mod, torch.zeros(1, b - a, heads * dim), freqs[:, a:b])
                out = wan_model.sequence_attention(mod, q, k, v)
            counters = {key: state[key] for key in ("kv_collectives", "kv_gathered_bytes", "out_collectives",
                                                    "out_exchanged_bytes", "padded_heads", "effective_comm_dtype")}
            return dict(bounds=(a, b), out=out, counters=counters)
        with emulated_collectives(world) as run:
            per_rank = run(rank_fn)
        (scases if mode == "ulysses" else tcases).append(dict(world=world, heads=heads, total=n_total, dim=dim,
                                                              ranks=per_rank))
    torch.save(dict(q_lin=q_lin, k_lin=k_lin, v_lin=v_lin, wq=wq, wk=wk, freqs=freqs, eps=1e-6,
                    cases=scases), HERE / "sequence_attention.pt")
    torch.save(dict(q_lin=q_lin, k_lin=k_lin, v_lin=v_lin, wq=wq, wk=wk, freqs=freqs, eps=1e-6,
                    cases=tcases), HERE / "sequence_attention_token.pt")
    # ------------------------------------------- self_attention_forward (B=2)
    from powershard.operations import Linear
    batch, n_total, heads, dim = 2, 300, 4, 128
    hidden = heads * dim
    g = torch.Generator().manual_seed(29)
    x = torch.randn(batch, n_total, hidden, generator=g)
    weights = [torch.randn(hidden, hidden, generator=g) * 0.02 for _ in range(4)]
    biases = [torch.randn(hidden, generator=g) * 0.01 for _ in range(4)]
    wq = torch.rand(hidden, generator=g) + 0.5
    wk = torch.rand(hidden, generator=g) + 0.5
    freqs = rope_table(n_total, dim // 2, 13)
    fcases = []
    for world in (1, 2):
        cfg = DistributedConfig(attention_backend="math", sequence_mode="ulysses")

        def rank_fn(rank):
            a, b = shard_bounds(n_total, rank, world) if world > 1 else (0, n_total)
            lin = []
            for w, bias in zip(weights, biases):
                layer = Linear(hidden, hidden, bias=True)
                layer.weight.data.copy_(w)
                layer.bias.data.copy_(bias)
                lin.append(layer)
            norm_q, norm_k = RMSNorm(hidden, eps=1e-6), RMSNorm(hidden, eps=1e-6)
            norm_q.weight.data.copy_(wq)
            norm_k.weight.data.copy_(wk)
            state = wan_model.new_sequence_state(cfg)
            state.update(total=n_total, enabled=world > 1, kv_collectives=0, kv_gathered_bytes=0,
                         out_collectives=0, out_exchanged_bytes=0, padded_heads=0, scale_collectives=0)
            mod = SimpleNamespace(num_heads=heads, head_dim=dim, norm_q=norm_q, norm_k=norm_k,
                                  q=lin[0], k=lin[1], v=lin[2], o=lin[3], _ps_qk_scales=(1., 1., 1.),
                                  _ps_sequence=state, _ps_attention=AttentionDispatcher(cfg),
                                  _ps_group="wan_self", _ps_safe=False)
            with torch.no_grad():
                out = wan_model.self_attention_forward(mod, x[:, a:b], freqs[:, a:b])
            counters = {key: state[key] for key in ("kv_collectives", "kv_gathered_bytes", "out_collectives",
                                                    "out_exchanged_bytes", "padded_heads")}
            return dict(bounds=(a, b), out=out, counters=counters)
        if world == 1:
            per_rank = [rank_fn(0)]
        else:
            with emulated_collectives(world) as run:
                per_rank = run(rank_fn)
        fcases.append(dict(world=world, ranks=per_rank))
    torch.save(dict(x=x, weights=weights, biases=biases, wq=wq, wk=wk, freqs=freqs, heads=heads, eps=1e-6,
                    cases=fcases), HERE / "self_attention_forward.pt")

    # ------------------------------------------------------ WanBackend.call
    from powershard import wan_backend
    bcases = []
    n_tok, n_blocks, heads = 96, 2, 2
    hidden = heads * dim
    g = torch.Generator().manual_seed(37)
    xw = torch.randn(1, n_tok, hidden, generator=g)
    bweights = [[torch.randn(hidden, hidden, generator=g) * 0.02 for _ in range(4)] for _ in range(n_blocks)]
    bnorm = [(torch.rand(hidden, generator=g) + 0.5, torch.rand(hidden, generator=g) + 0.5) for _ in range(n_blocks)]
    bfreqs = rope_table(n_tok, dim // 2, 17)
    saved_sharded = wan_backend.assert_sharded
    wan_backend.assert_sharded = lambda root, cpu_offload=None: None  # the stand-in root holds no FSDP shards
    try:
        for mode in ("ulysses", "token"):
            world = 2
            cfg = DistributedConfig(attention_backend="math", sequence_mode=mode)

            def rank_fn(rank):
                state = wan_model.new_sequence_state(cfg)
                blocks = []
                for ws, (wq_, wk_) in zip(bweights, bnorm):
                    lin = []
                    for w in ws:
                        layer = Linear(hidden, hidden, bias=True)
                        layer.weight.data.copy_(w)
                        layer.bias.data.zero_()
                        lin.append(layer)
                    norm_q, norm_k = RMSNorm(hidden, eps=1e-6), RMSNorm(hidden, eps=1e-6)
                    norm_q.weight.data.copy_(wq_)
                    norm_k.weight.data.copy_(wk_)
                    blocks.append(SimpleNamespace(num_heads=heads, head_dim=dim, norm_q=norm_q, norm_k=norm_k,
                                                  q=lin[0], k=lin[1], v=lin[2], o=lin[3], _ps_qk_scales=(1., 1., 1.),
                                                  _ps_sequence=state, _ps_attention=AttentionDispatcher(cfg),
                                                  _ps_group="wan_self", _ps_safe=False))

                def forward(x):
                    # The sequence handling of wan_forward (wan_model.py:1004-1011, :1073-1075).
                    total = x.shape[1]
                    state.update(total=total, enabled=world > 1, kv_collectives=0, kv_gathered_bytes=0,
                                 out_collectives=0, out_exchanged_bytes=0, scale_collectives=0, head_gathers=0)
                    a, b = shard_bounds(total, rank, world)
                    local = x[:, a:b]
                    for blk in blocks:
                        local = local + wan_model.self_attention_forward(blk, local, bfreqs[:, a:b])
                    out = wan_model.gather_tokens(local, total)
                    state["head_gathers"] += 1
                    return out

                class Root:
                    network = SimpleNamespace(blocks=blocks, num_heads=heads)

                    def __call__(self, command, args, kwargs):
                        return forward(*args)

                    def modules(self):
                        return iter(())

                    def named_modules(self):
                        return iter(())

                    def named_parameters(self):
                        return iter(())

                stub = lambda **kw: SimpleNamespace(**kw)  # noqa: E731
                backend = stub(
                    device=torch.device("cpu"), slot="main", world=world, sequence=state, root=Root(), units=[],
                    config=stub(reserve_gib=0.0, backend="fsdp2_sequence", cpu_offload=False, weight_placement="gpu"),
                    plan_memory=lambda args: dict(effective_prefetch=0),
                    ledger=stub(reset=lambda: None, report=lambda: {}),
                    tracker=stub(begin=lambda device: None, finish=lambda result: None),
                    attention=stub(report=lambda: {}), identity={}, lora_report=[],
                    spectrum=stub(report=lambda: {}), managed_pool=None, shard_bytes=0, buffer_bytes=0,
                    group_bytes=[0], options=stub(fp16_safe=False))
                with torch.no_grad():
                    out, metrics = wan_backend.WanBackend.call(backend, "forward", (xw,), {})
                keep = ("total", "enabled", "ulysses", "kv_collectives", "kv_gathered_bytes", "out_collectives",
                        "out_exchanged_bytes", "scale_collectives", "head_gathers", "padded_heads",
                        "effective_comm_dtype")
                return dict(out=out, state={k: state[k] for k in keep if k in state},
                            sequence_communication=metrics["sequence_communication"],
                            local_token_range=metrics["local_token_range"])
            with emulated_collectives(world) as run:
                per_rank = run(rank_fn)
            bcases.append(dict(mode=mode, world=world, ranks=per_rank))
    finally:
        wan_backend.assert_sharded = saved_sharded
    torch.save(dict(x=xw, weights=bweights, norms=bnorm, freqs=bfreqs, heads=heads, eps=1e-6, cases=bcases),
               HERE / "wan_backend_call.pt")

    # ---------------------------------------- image Layout SequenceAttention
    from powershard import image_parallel
    from powershard.image_layout import Layout

    def dense(q, k, v, heads, mask=None, skip_reshape=False, **kwargs):
        """Stand-in for ComfyUI optimized_attention: q/k/v [B,H,L,D] with
        skip_reshape, else [B,L,H*D]; returns [B,Lq,H*D] (fp32 math)."""
        if not skip_reshape:
            b, _, width = q.shape
            q, k, v = (t.view(b, -1, heads, width // heads).transpose(1, 2) for t in (q, k, v))
        o = torch.nn.functional.scaled_dot_product_attention(q.float(), k.float(), v.float())
        return o.transpose(1, 2).reshape(o.shape[0], o.shape[2], -1).to(q.dtype)

    icases = []
    for segments, world, batch, skip in (([(5, False), (13, True)], 2, 1, True),
                                         ([(5, False), (13, True)], 3, 2, False),
                                         ([(5, False), (13, True)], 5, 1, True),
                                         ([(4, False), (11, True), (3, False)], 3, 1, True)):
        heads, dim = 3, 16
        total = sum(n for n, _ in segments)
        gen = torch.Generator().manual_seed(31 + world)
        q, k, v = (torch.randn(batch, heads, total, dim, generator=gen) for _ in range(3))

        def rank_fn(rank):
            lay = Layout(segments, world, rank)
            stats = {}
            local = [image_parallel.localize(t, lay, 2) for t in (q, k, v)]
            if not skip:
                local = [t.transpose(1, 2).reshape(batch, t.shape[2], heads * dim) for t in local]
            sa = image_parallel.SequenceAttention(lay, stats)
            with torch.no_grad():
                out = sa(dense, *local, heads, skip_reshape=skip)
            return dict(out=out, sizes=list(lay.sizes), local_ranges=lay.local_ranges(), local_len=lay.local_len,
                        chunk=lay.chunk, stats=dict(stats))
        with emulated_collectives(world) as run:
            per_rank = run(rank_fn)
        icases.append(dict(segments=segments, world=world, heads=heads, skip_reshape=skip, q=q, k=k, v=v,
                           ranks=per_rank))
    torch.save(icases, HERE / "image_sequence_attention.pt")

    sizes = {p.name: p.stat().st_size for p in HERE.glob("*.pt")}
    print("wrote", sizes)


if __name__ == "__main__":
    main()
