"""The C ABI library: it loads, exports every symbol include/ps_b200.h
declares, and rejects invalid or unsupported requests with the documented
codes before touching the GPU (these calls need no device)."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def header_symbols():
    text = (ROOT / "include" / "ps_b200.h").read_text()
    return sorted(set(re.findall(r"\b(ps_b200_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from powershard_b200 import _lib, build_lib
    build_lib.build()
    return _lib.load()


def test_exports_every_header_symbol(lib):
    from powershard_b200 import _lib
    names = header_symbols()
    assert names, "no ps_b200_* declarations found in the header"
    for name in names:
        assert hasattr(lib, name), f"{name} not exported"
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"
    assert set(_lib.SIGNATURES) == set(names)


def test_abi_version(lib):
    from powershard_b200 import _lib
    assert lib.ps_b200_abi_version() == _lib.ABI_VERSION == 4
    assert lib.ps_b200_kernel_launches() == 0  # nothing launched without a GPU


def test_unsupported_dtype_is_reported_before_launch(lib):
    from powershard_b200 import _lib
    strides = _lib.i64([0, 0, 0])
    rc = lib.ps_b200_prepass(None, None, None, strides, None, None, None, 0, None, 0, None, _lib.FP32,
                             1, 0, 0, 1, 1, 128, 1e-6, 1, 0, 64, None)
    assert rc == _lib.ERR_UNSUPPORTED
    assert b"bf16" in lib.ps_b200_last_error()


def test_unsupported_head_dim(lib):
    from powershard_b200 import _lib
    st = _lib.i64([0, 0, 128, 64])
    rc = lib.ps_b200_attn_fwd(16, st, 16, st, 16, st, 16, st, _lib.BF16, _lib.BF16, 1, 1, 1, 64,
                              4, 1, 4, 4, 1, 4, 0.1, None, 0, None, None)
    assert rc == _lib.ERR_UNSUPPORTED
    assert b"head_dim" in lib.ps_b200_last_error()


def test_invalid_geometry(lib):
    from powershard_b200 import _lib
    # heads_per_rank * world < heads
    rc = lib.ps_b200_unpack(16, 16, 128, _lib.BF16, _lib.BF16, 2, 1, 1, 5, 2, 128, None)
    assert rc == _lib.ERR_INVALID
    # empty key set with queries
    st = _lib.i64([0, 0, 128, 128])
    rc = lib.ps_b200_attn_fwd(16, st, 16, st, 16, st, 16, st, _lib.BF16, _lib.BF16, 1, 1, 1, 128,
                              4, 1, 4, 4, 1, 0, 0.1, None, 0, None, None)
    assert rc == _lib.ERR_INVALID
    # misaligned pointer
    rc = lib.ps_b200_attn_fwd(18, st, 16, st, 16, st, 16, st, _lib.BF16, _lib.BF16, 1, 1, 1, 128,
                              4, 1, 4, 4, 1, 4, 0.1, None, 0, None, None)
    assert rc == _lib.ERR_INVALID
    assert b"aligned" in lib.ps_b200_last_error()


def test_segment_row_table_is_validated(lib):
    """The per-segment row table (image Layout balanced split) must hold
    `world` entries within [0, seg_rows] summing to total; it is checked on
    the host before anything touches the device."""
    from powershard_b200 import _lib
    ok = _lib.i32([3, 3, 2])  # split_sizes(8, 3)
    assert lib.ps_b200_ulysses_attn_fwd(16, 16, _lib.BF16, _lib.BF16, 3, 3, 8, ok, 2, 0, 128, 0.1,
                                        None, 0, None, None) == _lib.OK  # no valid heads: nothing to launch
    for bad, total in (([3, 3, 3], 8), ([4, 2, 2], 8), ([3, -1, 6], 8)):
        rc = lib.ps_b200_ulysses_attn_fwd(16, 16, _lib.BF16, _lib.BF16, 3, 3, total, _lib.i32(bad), 2, 2, 128,
                                          0.1, None, 0, None, None)
        assert rc == _lib.ERR_INVALID, bad
    rc = lib.ps_b200_ulysses_joint_attn_fwd(16, 16, 16, 16, _lib.BF16, _lib.BF16, 3, 3, 8, 4, _lib.i32([4, 2, 2]),
                                            2, 2, 128, 0.1, None, 0, None, None)
    assert rc == _lib.ERR_INVALID
    assert b"segment" in lib.ps_b200_last_error()


def test_empty_work_is_a_no_op(lib):
    from powershard_b200 import _lib
    st = _lib.i64([0, 0, 128, 128])
    assert lib.ps_b200_attn_fwd(16, st, 16, st, 16, st, 16, st, _lib.BF16, _lib.BF16, 1, 1, 1, 128,
                                4, 1, 0, 4, 1, 4, 0.1, None, 0, None, None) == _lib.OK
    assert lib.ps_b200_ulysses_attn_fwd(16, 16, _lib.BF16, _lib.BF16, 2, 3, 0, None, 2, 2, 128, 0.1, None, 0, None, None) == _lib.OK


def test_error_mapping_to_reference_exceptions():
    from powershard_b200 import _lib
    from powershard_b200.contract import UnsupportedAttention
    lib = _lib.load()
    rc = lib.ps_b200_unpack(16, 16, 128, _lib.FP32, _lib.FP32, 1, 1, 1, 1, 1, 128, None)
    with pytest.raises(UnsupportedAttention):
        _lib.check(rc, "unpack")
    rc = lib.ps_b200_unpack(16, 16, 128, _lib.BF16, _lib.BF16, 2, 1, 1, 5, 2, 128, None)
    with pytest.raises(ValueError):
        _lib.check(rc, "unpack")


def test_peer_and_token_entries_validate_on_the_host(lib):
    """The peer-store entry points reject bad tables and sizes before any
    device work (no GPU needed to see it)."""
    from powershard_b200 import _lib
    st = _lib.i64([128, 128, 128])
    # token fan-out: destination count out of range, null destinations
    rc = lib.ps_b200_prepass_token_to(16, 16, 16, st, None, 0, 0, _lib.BF16, 0, 0, 16, _lib.ptrs([16]), 0,
                                      _lib.BF16, 1, 1, 1, 128, 1e-6, 0, 0, 64, None)
    assert rc == _lib.ERR_INVALID
    rc = lib.ps_b200_prepass_token_to(16, 16, 16, st, None, 0, 0, _lib.BF16, 0, 0, 16, _lib.ptrs([16, 0]), 2,
                                      _lib.BF16, 1, 1, 1, 128, 1e-6, 0, 0, 64, None)
    assert rc == _lib.ERR_INVALID and b"destination 1" in lib.ps_b200_last_error()
    # broadcast: size not a multiple of 16, misaligned destination
    assert lib.ps_b200_broadcast(_lib.ptrs([16]), 1, 16, 24, None) == _lib.ERR_INVALID
    assert lib.ps_b200_broadcast(_lib.ptrs([18]), 1, 16, 32, None) == _lib.ERR_INVALID
    assert lib.ps_b200_broadcast(_lib.ptrs([16]), 1, 16, 0, None) == _lib.OK  # nothing to copy
    # joint attention to peer blocks: null table, row stride too small
    rc = lib.ps_b200_ulysses_joint_attn_to(16, 16, None, 256, 16, _lib.BF16, _lib.BF16, 2, 8, 16, 4, None,
                                           2, 2, 128, 0.1, None, 0, None, None)
    assert rc == _lib.ERR_INVALID
    rc = lib.ps_b200_ulysses_joint_attn_to(16, 16, _lib.ptrs([16, 16]), 128, 16, _lib.BF16, _lib.BF16, 2, 8, 16, 4,
                                           None, 2, 2, 128, 0.1, None, 0, None, None)
    assert rc == _lib.ERR_INVALID and b"row stride" in lib.ps_b200_last_error()
    # strided unpack: misaligned strides
    assert lib.ps_b200_unpack_strided(16, 12, 256, 16, 256, _lib.BF16, _lib.BF16, 4, 2, 1, 128,
                                      None) == _lib.ERR_INVALID
    # split-half RoPE geometry
    rc = lib.ps_b200_prepass(16, 16, 16, st, None, 16, 16, _lib.BF16, 16, 256, 16, _lib.BF16, 1, 4, 4, 1, 1, 128,
                             1e-6, 2, 1, 12, None)
    assert rc == _lib.ERR_UNSUPPORTED and b"split-half" in lib.ps_b200_last_error()


def test_static_block_rejects_head_dim_before_any_work(lib):
    """The allocation-free block computes head_dim 128 only; another head size
    is refused on the host, before the shared scratch is looked up or any work
    is queued on it."""
    from powershard_b200 import _lib
    rc = lib.ps_b200_block_fwd_static(16, 16, 16, _lib.i64([64, 64, 64]), 16, 16, _lib.FP32, 16, 128, 16,
                                      _lib.BF16, _lib.BF16, 100, 1, 64, 1e-6, 0.125, None, None)
    assert rc == _lib.ERR_UNSUPPORTED
    assert b"head_dim 128" in lib.ps_b200_last_error()
    assert lib.ps_b200_kernel_launches() == 0


def test_projection_entries_validate_on_the_host(lib):
    """The projection GEMM entries (powershard/wan_model.py:425-438 fused with
    the pre-pass and the unpack) refuse unsupported shapes and bad tables with
    the documented codes before any device work."""
    from powershard_b200 import _lib

    def qkv(dtype=_lib.BF16, batch=1, world=2, n_local=100, seg_rows=100, heads=4, hpr=2, head_dim=128, fin=256,
            eps=1e-6, dst=(16, 16)):
        table = _lib.ptrs(list(dst)) if dst is not None else None
        return lib.ps_b200_qkv_proj_batch(16, fin, 16, 16, 16, None, None, None, _lib.FP32, 16, 16, _lib.FP32, 16,
                                          0, 256, table, dtype, batch, world, n_local, seg_rows, heads, hpr,
                                          head_dim, fin, eps, None, 0, None, None)

    assert qkv(dtype=_lib.FP32) == _lib.ERR_UNSUPPORTED and b"bf16" in lib.ps_b200_last_error()
    assert qkv(head_dim=64) == _lib.ERR_UNSUPPORTED and b"head_dim 128" in lib.ps_b200_last_error()
    assert qkv(heads=3, hpr=2) == _lib.ERR_UNSUPPORTED and b"even head count" in lib.ps_b200_last_error()
    assert qkv(fin=100) == _lib.ERR_UNSUPPORTED and b"multiple of 64" in lib.ps_b200_last_error()
    assert qkv(heads=6, hpr=2) == _lib.ERR_INVALID  # 2 ranks x 2 heads cannot hold 6 heads
    assert qkv(seg_rows=50) == _lib.ERR_INVALID  # a segment shorter than the local rows
    assert qkv(eps=-1.0) == _lib.ERR_INVALID
    assert qkv(dst=None) == _lib.ERR_INVALID and b"destination table" in lib.ps_b200_last_error()
    assert qkv(dst=(16, 24)) == _lib.ERR_INVALID and b"destination block 1" in lib.ps_b200_last_error()
    assert qkv(batch=0) == _lib.OK  # nothing to do
    assert lib.ps_b200_qkv_proj_workspace_bytes(100, 4, 128) > 0

    def out(n_local=100, fin=256, fout=256, out_stride=256, block_cols=0, out_dtype=_lib.BF16):
        return lib.ps_b200_out_proj(16, fin, 0, block_cols, 16, None, _lib.FP32, 16, out_stride, _lib.BF16,
                                    out_dtype, n_local, fin, fout, None, None)

    assert out(fout=300) == _lib.ERR_UNSUPPORTED and b"out_features" in lib.ps_b200_last_error()
    assert out(out_dtype=_lib.FP16) == _lib.ERR_UNSUPPORTED
    assert out(out_stride=128) == _lib.ERR_INVALID
    assert out(block_cols=100) == _lib.ERR_UNSUPPORTED and b"multiple of 64" in lib.ps_b200_last_error()
    assert out(n_local=0) == _lib.OK
    assert lib.ps_b200_kernel_launches() == 0
