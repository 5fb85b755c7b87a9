"""Device-side failure detection without a GPU fault: a bounded wait that can
never complete must time out, record its status and return; the context stays
usable afterwards."""
import ctypes
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_reports(cuda_device):
    from ferret_b200 import _lib, ops
    L = _lib.lib()
    assert ops.last_device_status() == 0
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    t0 = time.perf_counter()
    assert L.ferret_selftest_wait_timeout(2_000_000, stream) == 0      # 2 ms
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 5.0
    st = ops.last_device_status()
    assert st & 0xFF == 1 and (st >> 8) & 0xFF == 15
    assert ops.last_device_status() == 0                               # cleared
    # the context is still healthy: a normal op runs and is correct
    x = torch.randn(8, 256, device="cuda").to(torch.bfloat16)
    q, s = ops.per_token_cast_to_fp8(x)
    torch.cuda.synchronize()
    assert torch.isfinite(s).all()


def test_selftest_rejects_unbounded_timeout(cuda_device):
    from ferret_b200 import _lib
    assert _lib.lib().ferret_selftest_wait_timeout(0, None) == -1
