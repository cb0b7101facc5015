"""Failure detection on the GPU without a fault: a bounded wait that nothing
satisfies expires, reports its code in the device status word, and the
context keeps working (a normal attention launch afterwards is correct)."""
import time

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def test_bounded_wait_expires_and_reports(cuda_lib):
    from powershard_b200 import _lib
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    start = time.time()
    _lib.check(cuda_lib.ps_b200_selftest_bounded_wait(status.data_ptr(), 50000,
                                                      torch.cuda.current_stream(DEV).cuda_stream), "selftest")
    torch.cuda.synchronize(DEV)
    assert time.time() - start < 5
    assert int(status.item()) == 199


def test_device_status_raises_on_host(cuda_lib):
    from powershard_b200 import _lib, ops
    st = ops.DeviceStatus(DEV)
    _lib.check(cuda_lib.ps_b200_selftest_bounded_wait(st.ptr, 20000, torch.cuda.current_stream(DEV).cuda_stream),
               "selftest")
    with pytest.raises(RuntimeError, match="bounded wait expired"):
        st.check()
    assert int(st.word.item()) == 0  # cleared after reporting


def test_context_usable_after_expired_wait(cuda_lib):
    from powershard_b200.provider import B200Provider
    q = torch.randn(1, 300, 2, 128, device=DEV, dtype=torch.bfloat16)
    out = B200Provider()(q, q, q)
    ref = torch.nn.functional.scaled_dot_product_attention(*(t.float().transpose(1, 2) for t in (q, q, q)))
    torch.testing.assert_close(out.float(), ref.transpose(1, 2), atol=2e-2, rtol=2e-2)
