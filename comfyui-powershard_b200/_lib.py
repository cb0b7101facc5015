"""ctypes binding of libps_b200.so, the C ABI declared in include/ps_b200.h.

The shared library is built in-tree (``lib/libps_b200.so`` next to this
file) by ``build_lib.build()``.  There is no fallback: a missing library, a
missing GPU or an unsupported device raises.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import torch

from .contract import UnsupportedAttention

LIB_PATH = Path(__file__).resolve().with_name("lib") / "libps_b200.so"
ABI_VERSION = 4

OK, ERR_INVALID, ERR_UNSUPPORTED, ERR_CUDA = 0, 1, 2, 3
BF16, FP16, FP32 = 0, 1, 2

# Every symbol of include/ps_b200.h with its ctypes signature.
_c_i64p = ctypes.POINTER(ctypes.c_int64)
_c_intp = ctypes.c_void_p
_c_ptrs = ctypes.POINTER(ctypes.c_void_p)  # void* const* (one pointer per rank)
SIGNATURES = {
    "ps_b200_abi_version": (ctypes.c_int, []),
    "ps_b200_last_error": (ctypes.c_char_p, []),
    "ps_b200_prepass": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, _c_i64p, _c_i64p,
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int64,
        ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
        ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]),
    "ps_b200_attn_fwd": (ctypes.c_int, [
        ctypes.c_void_p, _c_i64p, ctypes.c_void_p, _c_i64p, ctypes.c_void_p, _c_i64p,
        ctypes.c_void_p, _c_i64p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
        ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
        ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_void_p, ctypes.c_size_t, _c_intp, ctypes.c_void_p]),
    "ps_b200_ulysses_attn_fwd": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
        ctypes.c_int, ctypes.POINTER(ctypes.c_int), ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float,
        ctypes.c_void_p, ctypes.c_size_t, _c_intp, ctypes.c_void_p]),
    "ps_b200_block_fwd_static": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, _c_i64p, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.c_int, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
        ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_float,
        ctypes.POINTER(ctypes.c_int), ctypes.c_void_p]),
    "ps_b200_selftest_bounded_wait": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]),
    "ps_b200_ulysses_joint_attn_fwd": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
        ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_int), ctypes.c_int,
        ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_void_p, ctypes.c_size_t, _c_intp, ctypes.c_void_p]),
    "ps_b200_unpack": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int,
        ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]),
    "ps_b200_unpack_strided": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int,
        ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]),
    "ps_b200_prepass_to": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, _c_i64p, _c_i64p,
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int64,
        _c_ptrs, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
        ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]),
    "ps_b200_ulysses_attn_to": (ctypes.c_int, [
        ctypes.c_void_p, _c_ptrs, ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
        ctypes.c_int, ctypes.POINTER(ctypes.c_int), ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float,
        ctypes.c_void_p, ctypes.c_size_t, _c_intp, ctypes.c_void_p]),
    "ps_b200_shared_alloc": (ctypes.c_int, [ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p)]),
    "ps_b200_shared_free": (ctypes.c_int, [ctypes.c_void_p]),
    "ps_b200_ipc_export": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_ubyte)]),
    "ps_b200_ipc_import": (ctypes.c_int, [ctypes.POINTER(ctypes.c_ubyte), ctypes.POINTER(ctypes.c_void_p)]),
    "ps_b200_ipc_close": (ctypes.c_int, [ctypes.c_void_p]),
    "ps_b200_kernel_launches": (ctypes.c_ulonglong, []),
    "ps_b200_ulysses_joint_attn_to": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_void_p, _c_ptrs, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
        ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_int), ctypes.c_int,
        ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_void_p, ctypes.c_size_t, _c_intp, ctypes.c_void_p]),
    "ps_b200_broadcast": (ctypes.c_int, [_c_ptrs, ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]),
    "ps_b200_prepass_token_to": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, _c_i64p, _c_i64p,
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int64,
        ctypes.c_void_p, _c_ptrs, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
        ctypes.c_int, ctypes.c_float, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]),
    "ps_b200_prepass_batch": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, _c_i64p, _c_i64p, _c_i64p,
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
        _c_ptrs, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
        ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]),
    "ps_b200_ulysses_attn_batch": (ctypes.c_int, [
        ctypes.c_void_p, _c_ptrs, ctypes.c_int64, ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int,
        ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_int), ctypes.c_int, ctypes.c_int,
        ctypes.c_int, ctypes.c_float, ctypes.c_void_p, ctypes.c_size_t, _c_intp, ctypes.c_void_p]),
    "ps_b200_unpack_batch": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64,
        ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
        ctypes.c_int, ctypes.c_void_p]),
    "ps_b200_qkv_proj_workspace_bytes": (ctypes.c_size_t, [ctypes.c_int, ctypes.c_int, ctypes.c_int]),
    "ps_b200_qkv_proj": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.c_int, ctypes.c_void_p, ctypes.c_int64, _c_ptrs, ctypes.c_int, ctypes.c_int, ctypes.c_int,
        ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_void_p,
        ctypes.c_size_t, _c_intp, ctypes.c_void_p]),
    "ps_b200_qkv_proj_batch": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.c_int, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, _c_ptrs, ctypes.c_int, ctypes.c_int,
        ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
        ctypes.c_float, ctypes.c_void_p, ctypes.c_size_t, _c_intp, ctypes.c_void_p]),
    "ps_b200_out_proj": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.c_int, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
        ctypes.c_int, _c_intp, ctypes.c_void_p]),
}
ATTN_WORKSPACE_BYTES = 160 * 2 * 128 * 129 * 4
IPC_HANDLE_BYTES = 64

_LIB = None


class LibraryMissing(RuntimeError):
    """libps_b200.so is not built (run __graft_entry__.build() or build_lib.build())."""


def load():
    """Load the shared library once and attach the ctypes signatures."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not LIB_PATH.is_file():
        raise LibraryMissing(f"{LIB_PATH} is missing; build it with build_lib.build()")
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    if lib.ps_b200_abi_version() != ABI_VERSION:
        raise RuntimeError(f"libps_b200 ABI {lib.ps_b200_abi_version()} != {ABI_VERSION}")
    _LIB = lib
    return lib


def library_identity():
    """Stable fingerprint of the loaded library (path, size, mtime, ABI)."""
    stat = LIB_PATH.stat()
    return dict(module="powershard_b200", library=str(LIB_PATH), abi=ABI_VERSION,
                file_identity=[stat.st_size, stat.st_mtime_ns], arch="sm_100a")


def check(rc: int, what: str):
    """Map a C-ABI return code to the reference's exception contract.

    ERR_UNSUPPORTED -> UnsupportedAttention (the dispatcher may fall back);
    everything else -> ValueError / RuntimeError (never a silent fallback).
    """
    if rc == OK:
        return
    msg = (load().ps_b200_last_error() or b"").decode(errors="replace")
    if rc == ERR_UNSUPPORTED:
        raise UnsupportedAttention(f"{what}: {msg}")
    if rc == ERR_INVALID:
        raise ValueError(f"{what}: {msg}")
    raise RuntimeError(f"{what}: CUDA error: {msg}")


def dtype_code(dtype: torch.dtype) -> int:
    if dtype == torch.bfloat16:
        return BF16
    if dtype == torch.float16:
        return FP16
    if dtype == torch.float32:
        return FP32
    raise UnsupportedAttention(f"dtype {dtype} is not supported by the b200 kernels")


def i32(values):
    """ctypes int array of `values` (None stays None)."""
    if values is None:
        return None
    values = [int(v) for v in values]
    return (ctypes.c_int * len(values))(*values)


def ptrs(values):
    """ctypes void* array of device addresses (one per rank)."""
    values = [int(v) for v in values]
    return (ctypes.c_void_p * len(values))(*values)


def i64(values):
    return (ctypes.c_int64 * len(values))(*[int(v) for v in values])


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(t: torch.Tensor, what: str):
    if t.device.type != "cuda":
        raise UnsupportedAttention(f"{what}: the b200 kernels need CUDA tensors, got {t.device}")
