"""The C-ABI library: it loads, exports every symbol include/brew.h declares,
and validates arguments the way Linear.matmul does — without a GPU."""
import ctypes

import numpy as np
import pytest

from brewference_b200 import _native as N
from brewference_b200.api import Linear, PackedTensor
from brewference_b200 import config as C


def test_library_exports_every_declared_symbol():
    L = N.lib()
    syms = N.header_symbols()
    assert len(syms) >= 20
    missing = [s for s in syms if not hasattr(L, s)]
    assert not missing, missing


def test_type_geometry():
    L = N.lib()
    assert L.brew_type_bytes(C.TYPE_Q8_0, 64) == 68
    assert L.brew_type_bytes(C.TYPE_Q4_0, 64) == 36
    assert L.brew_type_bytes(C.TYPE_Q4_K, 512) == 288
    assert L.brew_type_bytes(C.TYPE_Q6_K, 256) == 210
    assert L.brew_type_bytes(C.TYPE_Q8_0, 33) == -1


def test_matmul_argument_validation_without_device():
    """Linear.validateMatmulArguments (Linear.java:67-74) fires before any
    device work, so it is checked here on the CPU."""
    out = np.zeros(4, np.float32)
    x = np.zeros(32, np.float32)
    rc = N.lib().brew_matmul(out.ctypes.data_as(N.c_f32p), x.ctypes.data_as(N.c_f32p), None, 0, 32, 4)
    assert rc == N.ERR_INVALID_ARG
    assert "Weight block cannot be null" in N.last_error()
    with pytest.raises(N.IllegalArgumentException):
        Linear.matmul(out, x, None, 0, 32, 4)


def test_no_cpu_fallback():
    """Without a CUDA device the library refuses to compute."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a device is present")
    with pytest.raises(N.NoDeviceError):
        N.init(0)
    with pytest.raises(N.BrewError):
        PackedTensor.upload(C.TYPE_Q8_0, np.zeros(34, np.uint8), 32)


def test_header_struct_layout():
    assert ctypes.sizeof(C.BrewConfig) == 25 * 4
