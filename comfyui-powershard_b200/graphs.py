"""CUDA graph capture of one attention call (engine, override or provider).

``GraphedCall(fn, *args, **kwargs)`` runs ``fn(*args, **kwargs)`` a few times
on a private stream (so the engine's per-stream buffers, attention workspace,
device status word and - on several ranks - the peer-exchange buffers exist
before capture), then captures one call into a ``torch.cuda.CUDAGraph`` on
the same stream.  ``graphed()`` replays it and returns the captured output
tensor; new inputs are written into the tensors given at capture time.

Every launch of the block is recorded once: the pre-pass, attention
(+ combine), unpack, the peer stores and - with more than one rank - the
4-byte NCCL all-reduces that order them, so a replay costs one graph launch
instead of a Python call per kernel.  Calls with more than one rank must be
captured and replayed on every rank in the same order.
"""
from __future__ import annotations

import torch


class GraphedCall:
    def __init__(self, fn, *args, warmup: int = 2, **kwargs):
        self.stream = torch.cuda.Stream()
        self.stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(self.stream):
            for _ in range(max(1, warmup)):
                fn(*args, **kwargs)
        self.stream.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=self.stream):
            self.out = fn(*args, **kwargs)
        torch.cuda.current_stream().wait_stream(self.stream)

    def __call__(self):
        """Replay on the current stream; returns the (static) output."""
        self.graph.replay()
        return self.out
