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
from brewference_b200.api import GemmPlan, PackedTensor

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


@pytest.mark.parametrize("qt", [C.TYPE_Q8_0, C.TYPE_Q4_0])
@pytest.mark.parametrize("T", [1, 50, 96])
def test_gemm_plan(device, qt, T):
    """A plan (the matrix repacked once, Q8_0 or Q4_0) run at token counts
    that are not multiples of the 32-token tile: rows past T stay untouched;
    a second, larger run grows the scratch."""
    K, Nr = 1024, 384
    w = oracle.synth_quantized(qt, 55, 4, Nr * K)
    t = PackedTensor.upload(qt, w, Nr * K)
    plan = GemmPlan(t, 0, K, Nr)
    for tt in (T, T + 40):
        x = np.random.default_rng(tt).standard_normal((tt, K)).astype(np.float32)
        xd = torch.from_numpy(x).cuda()
        yd = torch.full((tt + 3, Nr), float("nan"), dtype=torch.float32, device="cuda")
        plan.run(yd.data_ptr(), xd.data_ptr(), tt)
        torch.cuda.synchronize()
        y = yd.cpu().numpy()
        assert np.isnan(y[tt:]).all()
        for i in sorted({0, tt // 2, tt - 1}):
            assert rel(y[i], oracle.matvec(qt, w, 0, x[i], K, Nr)) < TOL, (tt, i)
    plan.free()
    t.free()


def test_gemm_plan_errors(device):
    w = oracle.synth_quantized(C.TYPE_Q4_K, 5, 2, 256 * 128)
    t = PackedTensor.upload(C.TYPE_Q4_K, w, 256 * 128)
    with pytest.raises(N.BrewError) as e:
        GemmPlan(t, 0, 256, 128)
    assert e.value.code == N.ERR_UNSUPPORTED
    t.free()
    w = oracle.synth_quantized(C.TYPE_Q8_0, 5, 2, 256 * 128)
    t = PackedTensor.upload(C.TYPE_Q8_0, w, 256 * 128)
    with pytest.raises(N.IllegalArgumentException):
        GemmPlan(t, 0, 256, 100)          # N not a multiple of 128
    with pytest.raises(N.IllegalStateException):
        GemmPlan(t, 256, 256, 128)        # past the tensor end
    t.free()
