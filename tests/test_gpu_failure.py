"""Failure detection on the GPU without a fault: every spin-wait of the
library's kernels is bounded.  brew_selftest_wait_timeout runs the two wait
forms the pipelines use (an mbarrier phase for the weight ring, the grid
barrier's arrival counter) against events that never happen, with a limit of
a few milliseconds: both must give up, the host must read BREW_ERR_TIMEOUT,
and the context must stay usable (a matvec afterwards is correct)."""
import ctypes
import time

import numpy as np
import pytest

import oracle
from brewference_b200 import _native as N
from brewference_b200 import config as C
from brewference_b200.api import Linear, PackedTensor

pytestmark = pytest.mark.gpu


def selftest(limit_ns):
    ended = ctypes.c_int32(-1)
    t0 = time.perf_counter()
    rc = N.lib().brew_selftest_wait_timeout(limit_ns, ctypes.byref(ended))
    return rc, ended.value, time.perf_counter() - t0


def test_bounded_waits_time_out_and_the_context_survives(device):
    for _ in range(2):   # repeatable: the error word is cleared by the read
        rc, ended, dt = selftest(5_000_000)
        assert rc == N.ERR_TIMEOUT, (rc, N.last_error())
        assert "timed out" in N.last_error()
        assert ended == 2
        assert dt < 5.0
    K, Nr = 512, 256
    w = oracle.synth_quantized(C.TYPE_Q8_0, 3, 1, Nr * K)
    t = PackedTensor.upload(C.TYPE_Q8_0, w, Nr * K)
    x = oracle.synth_fill(3, 2, 0, K, 1.0)
    y = np.zeros(Nr, np.float32)
    Linear.matmul(y, x, t, 0, K, Nr)
    ref = oracle.matvec(C.TYPE_Q8_0, w, 0, x, K, Nr)
    assert np.linalg.norm(y - ref) / np.linalg.norm(ref) < 1e-5
    t.free()


def test_limit_is_checked():
    assert N.lib().brew_selftest_wait_timeout(0, None) == N.ERR_INVALID_ARG
    assert N.lib().brew_selftest_wait_timeout(2_000_000_000, None) == N.ERR_INVALID_ARG
