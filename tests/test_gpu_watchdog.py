"""Failure detection on the GPU without a fault: a kernel whose bounded wait
can never be satisfied gives up after its budget, sets the device watchdog
word, and the host reads HEXCUDA_ERR_TIMEOUT; the device keeps working."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_watchdog_expiry_is_reported_and_device_stays_usable(hx, oracle):
    from hexkernels_b200 import _lib
    lib = _lib.load()
    assert lib.hexcuda_selftest_watchdog(0, 50) == 0
    rc = lib.hexcuda_sync(0)
    assert rc == 4, rc                       # HEXCUDA_ERR_TIMEOUT
    assert lib.hexcuda_last_error() == 4
    assert b"bounded device-side wait expired" in lib.hexcuda_last_error_string()
    # the word was cleared and the context is intact
    assert lib.hexcuda_sync(0) == 0
    x = np.random.default_rng(0).standard_normal((16, 4096)).astype(np.float32)
    np.testing.assert_allclose(hx.softmax(x), oracle.softmax(x), rtol=1e-5, atol=1e-7)


def test_watchdog_budget_is_validated(hx):
    from hexkernels_b200 import _lib
    lib = _lib.load()
    assert lib.hexcuda_selftest_watchdog(0, 0) == 1
    assert lib.hexcuda_selftest_watchdog(0, 5000) == 1
