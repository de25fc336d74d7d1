"""Failure detection on the device without a fault: a kernel whose bounded mbarrier wait can never
complete (nothing arrives on the barrier) gives up after a short budget, records MT_ERR_TIMEOUT in
the device status word and returns; the host reads the status, the context stays usable and the
next kernels run normally.  No test here faults, traps or hangs the GPU."""
import numpy as np
import pytest

import mtorch_b200 as mt
from mtorch_b200 import _lib

pytestmark = pytest.mark.gpu


def test_expired_wait_reports_timeout_and_context_survives():
    lib = _lib.lib()
    mt.cuda.synchronize()
    assert lib.mt_cuda_device_status(1) == _lib.MT_OK
    # ~10 ms at 2 GHz: the same bounded wait every pipelined kernel of the library uses
    _lib.check(lib.mt_cuda_selftest_wait_timeout(20_000_000, None), "wait self test")
    _lib.check(lib.mt_cuda_synchronize(None), "synchronize")
    assert lib.mt_cuda_device_status(0) == _lib.MT_ERR_TIMEOUT
    assert b"site 99" in lib.mt_cuda_last_error_string()
    with pytest.raises(RuntimeError):
        mt.cuda.synchronize()  # raises on the recorded timeout and clears it
    assert lib.mt_cuda_device_status(1) == _lib.MT_OK
    # the context is intact: a GEMM still runs and is right
    a = np.arange(64 * 32, dtype=np.float32).reshape(64, 32) / 1000
    b = np.ones((32, 16), np.float32)
    got = mt.matmul(mt.tensor(a).cuda(), mt.tensor(b).cuda()).numpy()
    np.testing.assert_allclose(got, a @ b, rtol=1e-5)


def test_wait_budget_is_bounded():
    lib = _lib.lib()
    assert lib.mt_cuda_selftest_wait_timeout(-1, None) == _lib.MT_ERR_INVALID
    assert lib.mt_cuda_selftest_wait_timeout(1 << 40, None) == _lib.MT_ERR_INVALID
