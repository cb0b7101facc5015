"""ps_b200_block_fwd_static: the single-GPU block for callers that may not
allocate device memory while they run (a plugin host that owns the device
memory budget through its own pool, or a step that must not trigger
cudaMalloc's implicit device synchronisation).

Called through the C ABI twice in a row with different inputs; each result
must match the existing entry points (ps_b200_prepass + ps_b200_ulysses_attn_fwd
at world size 1 with caller-allocated buffers) within the attention tolerance
of the other GPU tests, and the second call must leave the device's free
memory unchanged.  Kept in a file pytest collects last.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
MAX_ABS, MEAN_REL = 2e-2, 5e-3


def _inputs(n, heads, seed):
    from powershard_b200.rope import rope_table_3d
    g = torch.Generator(device=DEV).manual_seed(seed)
    x = [torch.randn(n, heads * 128, device=DEV, generator=g, dtype=torch.bfloat16) * 1.4 for _ in range(3)]
    wq = torch.rand(heads * 128, device=DEV, generator=g) + 0.5
    wk = torch.rand(heads * 128, device=DEV, generator=g) + 0.5
    freqs = rope_table_3d((n // 100 + 1, 10, 10), 128, device=DEV)[:n].contiguous()
    return x, wq, wk, freqs


def _static_call(lib, x, wq, wk, freqs, out, n, heads):
    from powershard_b200 import _lib
    status = ctypes.c_int(-1)
    rc = lib.ps_b200_block_fwd_static(
        x[0].data_ptr(), x[1].data_ptr(), x[2].data_ptr(), _lib.i64([t.stride(0) for t in x]),
        wq.data_ptr(), wk.data_ptr(), _lib.FP32, freqs.data_ptr(), freqs.stride(0), out.data_ptr(),
        _lib.BF16, _lib.BF16, n, heads, 128, 1e-6, 128 ** -0.5, ctypes.byref(status),
        torch.cuda.current_stream(DEV).cuda_stream)
    return rc, status.value


def _existing_path(lib, x, wq, wk, freqs, n, heads):
    from powershard_b200 import _lib
    stream = torch.cuda.current_stream(DEV).cuda_stream
    send = torch.empty((1, 3, n, heads, 128), device=DEV, dtype=torch.bfloat16)
    out = torch.empty((n, heads, 128), device=DEV, dtype=torch.bfloat16)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    _lib.check(lib.ps_b200_prepass(
        x[0].data_ptr(), x[1].data_ptr(), x[2].data_ptr(), _lib.i64([t.stride(0) for t in x]), None,
        wq.data_ptr(), wk.data_ptr(), _lib.FP32, freqs.data_ptr(), freqs.stride(0), send.data_ptr(), _lib.BF16,
        1, n, n, heads, heads, 128, 1e-6, 1, 0, 64, stream), "prepass")
    _lib.check(lib.ps_b200_ulysses_attn_fwd(send.data_ptr(), out.data_ptr(), _lib.BF16, _lib.BF16, 1, n, n, None,
                                            heads, heads, 128, 128 ** -0.5, None, 0, status.data_ptr(), stream), "attention")
    torch.cuda.synchronize(DEV)
    assert int(status.item()) == 0
    return out


def _assert_close(got, ref):
    got, ref = got.float(), ref.float()
    err = (got - ref).abs()
    rel = float(err.mean() / ref.abs().mean())
    assert float(err.max()) <= MAX_ABS and rel <= MEAN_REL, f"max_abs={float(err.max()):.3e} mean_rel={rel:.3e}"


def test_static_block_matches_existing_entry_points(cuda_lib):
    lib = cuda_lib
    n, heads = 1500, 6
    outs = [torch.empty((n, heads, 128), device=DEV, dtype=torch.bfloat16) for _ in range(2)]
    free_after_first = None
    for call, seed in enumerate((1, 2)):
        x, wq, wk, freqs = _inputs(n, heads, seed)
        ref = _existing_path(lib, x, wq, wk, freqs, n, heads)
        torch.cuda.synchronize(DEV)
        free_before = torch.cuda.mem_get_info(DEV)[0]
        rc, status = _static_call(lib, x, wq, wk, freqs, outs[call], n, heads)
        free_after = torch.cuda.mem_get_info(DEV)[0]
        assert rc == 0, lib.ps_b200_last_error()
        assert status == 0
        _assert_close(outs[call], ref)
        if call == 1:
            assert free_after == free_before, "the second call changed the device's free memory"
        free_after_first = free_after
    assert free_after_first is not None
    assert not torch.equal(outs[0], outs[1])


def test_static_block_rejects_sizes_beyond_its_scratch(cuda_lib):
    from powershard_b200 import _lib
    lib = cuda_lib
    n, heads = 131073, 1   # one token-head above the 96 MiB scratch
    rc = lib.ps_b200_block_fwd_static(16, 16, 16, _lib.i64([128, 128, 128]), 16, 16, _lib.FP32, 16, 256, 16,
                                      _lib.BF16, _lib.BF16, n, heads, 128, 1e-6, 0.1, None,
                                      torch.cuda.current_stream(DEV).cuda_stream)
    assert rc == _lib.ERR_UNSUPPORTED
    assert b"static scratch" in lib.ps_b200_last_error()
