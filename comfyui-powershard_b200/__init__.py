"""powershard_b200: B200 (sm_100a) Ulysses sequence-parallel attention for ComfyUI-PowerShard.

A drop-in ``b200`` attention provider and Wan self-attention path built on
hand-written CUDA kernels (libps_b200.so, C ABI in include/ps_b200.h):

* ``B200Provider`` - provider-API adapter (BLHD q/k/v -> output), the
  counterpart of powershard/attention_providers.py's adapters;
* ``UlyssesAttention`` - per-rank engine: fused q/k RMSNorm + RoPE + pack
  pre-pass, NCCL all-to-all, tcgen05/TMEM attention reading the receive
  buffer in place, all-to-all back, unpack;
* ``wan.self_attention_forward`` / ``wan.sequence_attention`` - the
  reference's Wan entry points (powershard/wan_model.py:433-502);
* ``image.SequenceAttention`` - the Flux block attention override
  (powershard/image_parallel.py:67-110) on the Ulysses exchange and the
  joint [text; image] kernel;
* ``probe`` - the provider certification probe (powershard/attention_probe.py).

The package directory doubles as a ComfyUI custom-node folder (it registers
no nodes; PowerShard selects the provider by ``attention_backend="b200"``).
"""
from .contract import AttentionOptions, UnsupportedAttention, validate
from .partition import ImageLayout, UlyssesGeometry, shard_bounds, split_sizes

NODE_CLASS_MAPPINGS: dict = {}
NODE_DISPLAY_NAME_MAPPINGS: dict = {}

__all__ = [
    "AttentionOptions", "UnsupportedAttention", "validate", "UlyssesGeometry", "shard_bounds",
    "ImageLayout", "split_sizes", "B200Provider", "UlyssesAttention", "SequenceAttention",
    "NODE_CLASS_MAPPINGS", "NODE_DISPLAY_NAME_MAPPINGS",
]


def __getattr__(name):  # lazy: importing the package never needs a GPU
    if name == "B200Provider":
        from .provider import B200Provider
        return B200Provider
    if name == "UlyssesAttention":
        from .ulysses import UlyssesAttention
        return UlyssesAttention
    if name == "SequenceAttention":
        from .image import SequenceAttention
        return SequenceAttention
    raise AttributeError(name)
