"""brew_matmul_dev_static (the device matvec whose scratch is a fixed module
array, so the call allocates nothing) against brew_matmul_dev on the same
inputs, through the C ABI.  Two calls in a row must each match the existing
entry point (same kernels, so the tolerance 1e-6 relative L2 is loose), and
an input too large for the fixed array is refused.  Collected last (file
name) so that it also runs after every other GPU test; it initialises the
library itself, so it passes alone too.
"""
import ctypes

import numpy as np
import pytest
import torch

import oracle
from brewference_b200 import _native as N
from brewference_b200 import config as C
from brewference_b200.api import Linear, PackedTensor

pytestmark = pytest.mark.gpu
TOL = 1e-6


def rel(a, b):
    a = a.astype(np.float64)
    b = b.astype(np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def static_matmul(y, x, t, off, K, Nout, batch, stream=0):
    return N.lib().brew_matmul_dev_static(y.data_ptr(), x.data_ptr(), t.handle, off, K, Nout, batch, stream)


@pytest.mark.parametrize("qt,K,Nout,batch", [(C.TYPE_Q8_0, 2048, 1536, 1), (C.TYPE_Q4_0, 1024, 520, 3),
                                             (C.TYPE_Q8_0, 4096, 256, 16), (C.TYPE_Q8_0, 512, 300, 20)])
def test_static_matches_dynamic(qt, K, Nout, batch):
    N.init(0)
    w = oracle.synth_quantized(qt, 5, 9, Nout * K)
    t = PackedTensor.upload(qt, w, Nout * K)
    rng = np.random.default_rng(3)
    x = torch.from_numpy(rng.standard_normal((batch, K)).astype(np.float32)).cuda()
    want = torch.zeros((batch, Nout), dtype=torch.float32, device="cuda")
    Linear.matmul_device(want.data_ptr(), x.data_ptr(), t, 0, K, Nout, batch)
    torch.cuda.synchronize()
    for _ in range(2):
        got = torch.full((batch, Nout), float("nan"), dtype=torch.float32, device="cuda")
        assert static_matmul(got, x, t, 0, K, Nout, batch) == 0, N.last_error()
        torch.cuda.synchronize()
        assert rel(got.cpu().numpy(), want.cpu().numpy()) < TOL
    t.free()


def test_static_refuses_oversized_input():
    N.init(0)
    K, Nout = 16384, 16
    w = oracle.synth_quantized(C.TYPE_Q8_0, 5, 10, Nout * K)
    t = PackedTensor.upload(C.TYPE_Q8_0, w, Nout * K)
    x = torch.zeros((16, K), dtype=torch.float32, device="cuda")
    y = torch.zeros((16, Nout), dtype=torch.float32, device="cuda")
    assert static_matmul(y, x, t, 0, K, Nout, 16) == N.ERR_INVALID_ARG
    assert "static scratch" in N.last_error()
    t.free()
