"""Ulysses exchange over NVLink peer memory (one process per GPU, one node).

The reference moves q/k/v and the attention output with two
``all_to_all_single`` calls per block (powershard/wan_model.py:360 and :376).
Here each rank instead owns two buffers that every rank of the group maps
into its address space (CUDA IPC):

* ``recv``    [W][3][B][width][h][D]: rank s's pre-pass stores its block for
  this rank at ``recv[s]`` directly over NVLink (``ps_b200_prepass_batch``);
* ``staging`` [B][width][W*h][D]: the attention kernel of rank r stores the
  output rows of this rank's tokens for heads [r*h, (r+1)*h) directly into
  ``staging[:, :, r*h:(r+1)*h]`` (``ps_b200_ulysses_attn_batch``);
* ``text`` [W][P][h][D] (joint attention only): rank r copies the text
  outputs of its heads into ``text[r]`` of every rank (``ps_b200_broadcast``),
  the all-gather over heads of the replicated text rows;
* token layout: one buffer ``kv_all`` [W][2][width][H][D]; rank r's
  pre-pass stores its k/v rows into slot r of every rank's buffer
  (``ps_b200_prepass_token_to``), the K/V all-gather of token mode.

So the transfers ride on the kernels' own stores and overlap their compute;
what remains for the host is ordering across ranks.  ``barrier()`` is a
4-byte NCCL all-reduce on the current stream.  On each rank it starts only
after the rank's previous kernel has completed - and a completed kernel's
stores, peer stores included, are visible at system scope - and it ends only
after every rank has joined, so after it every rank's previously enqueued
stores are visible everywhere.  One barrier between pre-pass and attention
makes the received blocks complete; one between attention and unpack makes
the staged outputs complete, and the pair also keeps a rank from
overwriting a buffer a peer still reads in the previous or next step.
"""
from __future__ import annotations

import ctypes
import math
import socket

import torch
import torch.distributed as dist

from . import _lib
from .partition import UlyssesGeometry


class _DeviceBuffer:
    """__cuda_array_interface__ view of raw device memory (no ownership)."""

    def __init__(self, ptr: int, numel: int):
        self.__cuda_array_interface__ = dict(shape=(numel,), typestr="<i2", data=(ptr, False), version=3,
                                             strides=None)


def _wrap(ptr: int, shape, dtype: torch.dtype, device: torch.device) -> torch.Tensor:
    numel = math.prod(shape)
    flat = torch.as_tensor(_DeviceBuffer(ptr, numel), device=device)
    return flat.view(dtype).view(shape)


class PeerExchange:
    """Shared receive / staging buffers of one geometry for the ranks of `group`.

    Build with ``PeerExchange.create`` (collective: every rank of the group
    calls it with the same geometry); it returns None on every rank when any
    rank cannot map its peers' memory, and the caller then keeps the NCCL
    all-to-all.
    """

    def __init__(self, group, geo: UlyssesGeometry, dtype: torch.dtype, device: torch.device, text_rows: int = 0,
                 layout: str = "ulysses", batch: int | None = None):
        self.group, self.geo, self.dtype, self.device = group, geo, dtype, device
        self.text_rows = int(text_rows)
        self.layout = layout
        self.batch = batch  # None: unbatched buffers [W][3][width][h][D] / [width][W*h][D]
        self.own = []         # device pointers this rank allocated
        self.imported = []    # device pointers mapped from peers
        self.recv_ptrs = []
        self.stage_ptrs = []
        self.flag = torch.zeros(1, dtype=torch.int32, device=device)
        self.closed = False

    # ------------------------------------------------------------ setup
    @classmethod
    def create(cls, group, geo: UlyssesGeometry, dtype: torch.dtype, device: torch.device, text_rows: int = 0,
               layout: str = "ulysses", batch: int | None = None):
        ex = cls(group, geo, dtype, device, text_rows, layout, batch)
        ok, reason = ex._setup()
        verdict = torch.tensor([1 if ok else 0], dtype=torch.int32, device=device)
        dist.all_reduce(verdict, op=dist.ReduceOp.MIN, group=group)
        if int(verdict.item()) != 1:
            ex._teardown()
            return None
        return ex

    def _setup(self):
        lib = _lib.load()
        geo = self.geo
        esize = self.dtype.itemsize
        h, d = geo.heads_per_rank, geo.head_dim
        if self.layout == "token":  # gathered K/V of every rank: [W][2][width][H][D]
            shapes = [(geo.world, 2, geo.width, geo.heads, d)]
        elif self.batch is not None:
            shapes = [geo.send_shape(self.batch), (self.batch, geo.width, geo.padded_heads, d)]
        else:
            shapes = [geo.send_shape(), (geo.width, geo.padded_heads, d)]
            if self.text_rows:
                shapes.append((geo.world, self.text_rows, h, d))
        nbytes = _lib.IPC_HANDLE_BYTES
        handles = bytearray()
        error = None
        try:
            with torch.cuda.device(self.device):
                for shape in shapes:
                    ptr = ctypes.c_void_p()
                    _lib.check(lib.ps_b200_shared_alloc(max(1, math.prod(shape)) * esize, ctypes.byref(ptr)),
                               "ps_b200_shared_alloc")
                    self.own.append(ptr.value)
                    hdl = (ctypes.c_ubyte * nbytes)()
                    _lib.check(lib.ps_b200_ipc_export(ptr.value, hdl), "ps_b200_ipc_export")
                    handles += bytes(hdl)
        except (RuntimeError, ValueError) as e:
            error = str(e)
            handles = bytearray(len(shapes) * nbytes)
        table = [None] * geo.world
        dist.all_gather_object(table, (socket.gethostname(), bytes(handles), error), group=self.group)
        if any(entry[2] for entry in table):
            return False, next(entry[2] for entry in table if entry[2])
        if len({entry[0] for entry in table}) != 1:
            return False, "ranks on more than one host"
        ptrs = [[] for _ in shapes]  # ptrs[buffer][rank]
        try:
            with torch.cuda.device(self.device):
                for r, (_, blob, _) in enumerate(table):
                    for part in range(len(shapes)):
                        if r == geo.rank:
                            ptrs[part].append(self.own[part])
                            continue
                        hdl = (ctypes.c_ubyte * nbytes).from_buffer_copy(blob[part * nbytes:(part + 1) * nbytes])
                        ptr = ctypes.c_void_p()
                        _lib.check(lib.ps_b200_ipc_import(hdl, ctypes.byref(ptr)), "ps_b200_ipc_import")
                        self.imported.append(ptr.value)
                        ptrs[part].append(ptr.value)
        except (RuntimeError, ValueError) as e:
            return False, str(e)
        if self.layout == "token":
            self.kv_all = _wrap(self.own[0], shapes[0], self.dtype, self.device)
            kv_block = 2 * geo.width * geo.heads * d * esize     # one rank's [2][width][H][D] slot
            self.kv_dst = [p + geo.rank * kv_block for p in ptrs[0]]
            return True, None
        self.recv_ptrs, self.stage_ptrs = ptrs[0], ptrs[1]
        self.recv = _wrap(self.own[0], shapes[0], self.dtype, self.device)
        self.staging = _wrap(self.own[1], shapes[1], self.dtype, self.device)
        nb = 1 if self.batch is None else self.batch
        block = 3 * nb * geo.width * h * d * esize              # one source's [3][B][width][h][D] block
        self.dst_blocks = [p + geo.rank * block for p in self.recv_ptrs]
        self.out_blocks = [p + geo.rank * h * d * esize for p in self.stage_ptrs]
        self.out_row_stride = geo.padded_heads * d
        self.out_batch_stride = geo.width * geo.padded_heads * d
        if self.text_rows:
            self.text = _wrap(self.own[2], shapes[2], self.dtype, self.device)
            tblock = self.text_rows * h * d * esize
            self.text_dst = [p + geo.rank * tblock for p in ptrs[2]]
        return True, None

    # ------------------------------------------------------------ per step
    def barrier(self):
        """Stream-ordered cross-rank barrier (4-byte NCCL all-reduce)."""
        dist.all_reduce(self.flag, group=self.group)

    # ------------------------------------------------------------ teardown
    def _teardown(self):
        """Collective: every rank unmaps its peers' buffers, then (after a
        barrier) frees its own."""
        torch.cuda.synchronize(self.device)
        lib = _lib.load()
        with torch.cuda.device(self.device):
            for p in self.imported:
                lib.ps_b200_ipc_close(p)
            self.imported = []
            if dist.get_backend(self.group) == "nccl":
                dist.barrier(group=self.group, device_ids=[self.device.index])
            else:
                dist.barrier(group=self.group)
            for p in self.own:
                lib.ps_b200_shared_free(p)
            self.own = []

    def close(self):
        """Release the shared buffers (collective over the group)."""
        if not self.closed:
            self.closed = True
            self._teardown()
