"""Worker-side integration of the b200 self-attention into a Wan network.

PowerShard's worker builds the Wan network, then ``install_wan_compute``
(powershard/wan_model.py:727-768) replaces each attention module's
``forward`` and attaches the shared sequence state ``net._ps_sequence``;
``wan_forward`` (wan_model.py:1004-1005, :1073-1075) resets that state's
counters every forward, and ``WanBackend.call`` (wan_backend.py:413-496)
reports them as ``metrics["sequence_communication"]`` (wan_backend.py:483-495).

* ``install_network(net, state=None, group=None)`` - the b200 counterpart of
  the ``"self"`` branch of ``install_wan_compute`` for a whole network: every
  WanSelfAttention-like module (q/k/v/o projections, norm_q/norm_k,
  num_heads/head_dim) gets ``wan.self_attention_forward`` and shares the
  network's sequence state, so ``wan_forward`` and ``WanBackend.call`` read
  the b200 counters unchanged.
* ``sequence_communication(state)`` - the metrics block ``WanBackend.call``
  builds from that state, for hosts that assemble their own report.
"""
from __future__ import annotations

from .wan import install_self_attention

_PROJECTIONS = ("q", "k", "v", "o", "norm_q", "norm_k")


def is_self_attention(module) -> bool:
    """A WanSelfAttention-like module: q/k/v/o projections, RMSNorm q/k and
    the head geometry install_wan_compute reads (wan_model.py:684-700)."""
    if getattr(module, "_ps_cross", False) or type(module).__name__.endswith("CrossAttention"):
        return False
    return all(hasattr(module, name) for name in _PROJECTIONS) and hasattr(module, "num_heads") \
        and hasattr(module, "head_dim")


def install_network(net, state: dict | None = None, group=None) -> list:
    """Route every self-attention module of ``net`` through the b200 path.

    ``state`` defaults to ``net._ps_sequence`` (created if absent); it is
    attached to ``net`` and to every routed module, as install_wan_compute
    does (wan_model.py:733-746).  Returns the names of the routed modules.
    """
    if state is None:
        state = getattr(net, "_ps_sequence", None)
        if state is None:
            state = dict(total=0, enabled=False, ulysses=True, comm_dtype="bf16", mode="ulysses")
    net._ps_sequence = state
    routed = []
    for name, module in net.named_modules():
        if module is not net and is_self_attention(module):
            install_self_attention(module, group, state)
            routed.append(name)
    return routed


def sequence_communication(state: dict) -> dict | None:
    """The ``sequence_communication`` metrics of one forward from the shared
    sequence state (the block of powershard/wan_backend.py:483-495); None when
    the forward ran without sequence parallelism."""
    if not state.get("enabled"):
        return None
    ulysses = state.get("ulysses", True)
    return dict(
        mode="ulysses" if ulysses else "token",
        communication_dtype=state.get("effective_comm_dtype"),
        kv_all_gathers=state.get("kv_collectives", 0) if not ulysses else 0,
        qkv_all_to_all=state.get("kv_collectives", 0) if ulysses else 0,
        output_all_to_all=state.get("out_collectives", 0),
        scale_all_reduces=state.get("scale_collectives", 0),
        exchanged_bytes=state.get("kv_gathered_bytes", 0) + state.get("out_exchanged_bytes", 0),
        head_output_all_gathers=state.get("head_gathers", 0),
        note="Logical tensor bytes, not measured NCCL link traffic")
