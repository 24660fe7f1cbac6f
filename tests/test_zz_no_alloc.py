"""brew_matmul_dev_static: the device matvec for callers that cannot allocate
device memory in the middle of a call (a JNI critical region, where the JVM
has pinned arrays and a blocking cudaMalloc would stall its garbage
collector, or a server that reserves all its device memory up front).  Its
scratch is a fixed array inside the loaded library, so the call allocates
nothing.

Checked through the C ABI, two calls in a row each time:
  * against the oracle's Linear.matmul (relative L2 1e-5, the tolerance of
    the other matvec tests) and against brew_matmul_dev (same kernels);
  * Q8_0, Q4_0 and a Q4_K case (the K-quant branch, which needs no scratch);
  * free device memory is unchanged across the calls after the first one;
  * an input too large for the fixed array is refused.
Collected last (file name) so that it runs after every other GPU test; it
initialises the library itself, so it passes alone too.
"""
import numpy as np
import pytest
import torch

import oracle
from brewference_b200 import _native as N
from brewference_b200 import config as C
from brewference_b200.api import Linear, PackedTensor

pytestmark = pytest.mark.gpu
TOL = 1e-5


def rel(a, b):
    a = a.astype(np.float64)
    b = b.astype(np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def static_matmul(y, x, t, off, K, Nout, batch, stream=0):
    return N.lib().brew_matmul_dev_static(y.data_ptr(), x.data_ptr(), t.handle, off, K, Nout, batch, stream)


@pytest.mark.parametrize("qt,K,Nout,batch", [(C.TYPE_Q8_0, 2048, 1536, 1), (C.TYPE_Q4_0, 1024, 520, 3),
                                             (C.TYPE_Q8_0, 4096, 256, 16), (C.TYPE_Q8_0, 512, 300, 20),
                                             (C.TYPE_Q4_K, 1024, 384, 2)])
def test_static_matches_oracle_and_dynamic(qt, K, Nout, batch):
    N.init(0)
    layers = 2   # the second layer's rows through the element offset
    w = oracle.synth_quantized(qt, 5, 9, layers * Nout * K)
    t = PackedTensor.upload(qt, w, layers * Nout * K)
    off = Nout * K
    rng = np.random.default_rng(3)
    xh = rng.standard_normal((batch, K)).astype(np.float32)
    x = torch.from_numpy(xh).cuda()
    want = np.stack([oracle.matvec(qt, w, off, xh[b], K, Nout) for b in range(batch)])
    dyn = torch.zeros((batch, Nout), dtype=torch.float32, device="cuda")
    Linear.matmul_device(dyn.data_ptr(), x.data_ptr(), t, off, K, Nout, batch)
    torch.cuda.synchronize()
    free0 = None
    for call in range(2):
        got = torch.full((batch, Nout), float("nan"), dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()
        if call == 1:
            free0 = torch.cuda.mem_get_info()[0]
        assert static_matmul(got, x, t, off, K, Nout, batch) == 0, N.last_error()
        torch.cuda.synchronize()
        if call == 1:
            assert torch.cuda.mem_get_info()[0] == free0, "the call changed free device memory"
        g = got.cpu().numpy()
        assert np.isfinite(g).all()
        assert rel(g, want) < TOL, (call, rel(g, want))
        assert rel(g, dyn.cpu().numpy()) < 1e-6, call
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
