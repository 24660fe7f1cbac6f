"""The prefill GEMM on the tcgen05 tensor cores (brew_gemm_q8_dev) against
the oracle's Java-order matvec, token by token: every output row within
1e-5 relative L2 (the integer block products are exact; fp32 accumulation
order differs), at a small and at a model-sized shape."""
import numpy as np
import pytest
import torch

import oracle
from brewference_b200 import _native as N
from brewference_b200 import config as C
from brewference_b200.api import PackedTensor

pytestmark = pytest.mark.gpu
TOL = 1e-5


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def gemm(t, off, K, Nr, x):
    T = x.shape[0]
    xd = torch.from_numpy(x).cuda()
    yd = torch.full((T, Nr), float("nan"), dtype=torch.float32, device="cuda")
    N.check(N.lib().brew_gemm_q8_dev(yd.data_ptr(), xd.data_ptr(), t.handle, off, K, Nr, T, None), "gemm")
    torch.cuda.synchronize()
    return yd.cpu().numpy()


@pytest.mark.parametrize("K,Nr,T,check", [(512, 256, 64, 64), (2048, 2048, 128, 6)])
def test_gemm_matches_oracle(device, K, Nr, T, check):
    w = oracle.synth_quantized(C.TYPE_Q8_0, 41, 2, Nr * K)
    t = PackedTensor.upload(C.TYPE_Q8_0, w, Nr * K)
    x = np.random.default_rng(7).standard_normal((T, K)).astype(np.float32)
    y = gemm(t, 0, K, Nr, x)
    for i in np.linspace(0, T - 1, check).astype(int):
        ref = oracle.matvec(C.TYPE_Q8_0, w, 0, x[i], K, Nr)
        assert rel(y[i], ref) < TOL, (i, rel(y[i], ref))
    t.free()


def test_gemm_weight_offset_and_errors(device):
    K, Nr, T = 256, 128, 32
    w = oracle.synth_quantized(C.TYPE_Q8_0, 43, 3, 2 * Nr * K)
    t = PackedTensor.upload(C.TYPE_Q8_0, w, 2 * Nr * K)
    x = np.random.default_rng(9).standard_normal((T, K)).astype(np.float32)
    y = gemm(t, Nr * K, K, Nr, x)                 # the second matrix of the tensor
    ref = oracle.matvec(C.TYPE_Q8_0, w, Nr * K, x[5], K, Nr)
    assert rel(y[5], ref) < TOL
    xd = torch.zeros((T, K), dtype=torch.float32, device="cuda")
    yd = torch.zeros((T, 100), dtype=torch.float32, device="cuda")
    assert N.lib().brew_gemm_q8_dev(yd.data_ptr(), xd.data_ptr(), t.handle, 0, K, 100, T, None) == N.ERR_INVALID_ARG
    t.free()
