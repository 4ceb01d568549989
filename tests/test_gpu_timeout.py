"""The device-side timeout path (every kernel's mbarrier waits are bounded): a wait that
nothing completes runs out after a few seconds, the kernel returns, the host call reports
ZWG_TIMEOUT through the error word, and the same context keeps working. The failure is made
by a barrier no thread ever arrives on (zwg_selftest_timeout); nothing faults or traps."""
import numpy as np
import pytest

from oracle import attention as A
from tests.conftest import has_gpu

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_timeout_and_context_survives():
    if not has_gpu():
        pytest.fail("needs a CUDA device")
    from zwhisper_b200 import _lib, ops
    _lib.ensure_init(0)
    lib = _lib.load()
    rc = lib.zwg_selftest_timeout()
    assert rc == _lib.ZWG_TIMEOUT, _lib.last_error()
    assert "timed out" in _lib.last_error()
    # the error word was cleared and the context is usable: an ordinary call succeeds
    assert lib.zwg_sync() == _lib.ZWG_OK
    rng = np.random.default_rng(0)
    q, k, v = (rng.random(n * 64, dtype=np.float32) - 0.5 for n in (5, 40, 40))
    got = ops.attention(q, k, v, 5, 40, 64, 2, True)
    want = A.attention(q, k, v, 5, 40, 64, 2, True)
    np.testing.assert_allclose(got, want, atol=1e-4, rtol=0)
