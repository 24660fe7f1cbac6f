"""GPU parity of the packed-block kernels against the oracle, through the C ABI.

Tolerances: dequantized weights are compared bit for bit; matvec outputs are
required to be within 1e-5 relative L2 of the oracle's Java-order fp32 sums
(the acceptance bar is 1e-3; the limb-MMA path is exact in the integer block
sums, so its error is at the fp32 rounding level).
"""
import numpy as np
import pytest
import torch

import oracle
from brewference_b200 import _native as native
from brewference_b200 import config as C
from brewference_b200.api import DeviceModel, Linear, PackedTensor

pytestmark = pytest.mark.gpu
TOL = 1e-5


def rel(a, b):
    return float(np.linalg.norm(a.astype(np.float64) - b) / max(np.linalg.norm(b.astype(np.float64)), 1e-30))


@pytest.mark.parametrize("qt", [C.TYPE_Q8_0, C.TYPE_Q4_0, C.TYPE_Q4_K, C.TYPE_Q6_K])
def test_dequantize_bit_exact(device, qt):
    n = 256 * 40
    w = oracle.synth_quantized(qt, 21, 3, n)
    t = PackedTensor.upload(qt, w, n)
    assert np.array_equal(t.read_bytes(), w)
    for off, m in ((0, n), (256, 512), (32 * 5, 96)):
        if qt in (C.TYPE_Q4_K, C.TYPE_Q6_K) and off % 256:
            continue
        d = t.dequantize_row(off, m)
        ref = oracle.dequantize(qt, w, off, m)
        assert np.array_equal(d.view(np.uint32), ref.view(np.uint32))


def test_device_synth_bytes_equal_oracle(device):
    cfg = C.smollm2_135m().replace(n_layers=2, vocab_size=1024)
    dm = DeviceModel.synthesize(cfg, 1234)
    om = oracle.OracleModel(cfg, 1234)
    for w in range(9):
        if w == C.W_OUTPUT:
            continue
        assert np.array_equal(dm.tensor(w).read_bytes(), om.tensor(w)), w


@pytest.mark.parametrize("qt", [C.TYPE_Q4_0, C.TYPE_Q4_K, C.TYPE_Q6_K])
def test_device_synth_other_types(device, qt):
    cfg = C.smollm2_135m().replace(n_layers=1, vocab_size=512, dim=512, hidden_dim=1024, n_heads=8, n_kv_heads=4,
                                   type_q=qt, type_k=qt, type_v=qt, type_o=qt, type_gate=qt, type_up=qt, type_down=qt)
    om = oracle.OracleModel(cfg, 77)
    # the device model refuses K-quant layers; generate the tensors alone
    t = PackedTensor.upload(qt, om.tensor(C.W_Q), cfg.q_width * cfg.dim)
    assert np.array_equal(t.read_bytes(), om.tensor(C.W_Q))


SHAPES = [(576, 192), (576, 1536), (1536, 576), (2048, 4096), (6144, 2048), (1152, 1024), (2048, 1),
          (2048, 7), (2048, 17), (4096, 100), (32, 3), (6912, 1152)]


@pytest.mark.parametrize("qt", [C.TYPE_Q8_0, C.TYPE_Q4_0])
@pytest.mark.parametrize("K,N", SHAPES)
def test_matmul_matches_oracle(device, qt, K, N):
    rng = np.random.default_rng(K * 7 + N)
    w = oracle.synth_quantized(qt, 5, K + N, K * N)
    t = PackedTensor.upload(qt, w, K * N)
    x = rng.standard_normal(K).astype(np.float32)
    y = np.empty(N, np.float32)
    Linear.matmul(y, x, t, 0, K, N)
    ref = oracle.matvec(qt, w, 0, x, K, N)
    assert rel(y, ref) < TOL, rel(y, ref)


@pytest.mark.parametrize("qt", [C.TYPE_Q4_K, C.TYPE_Q6_K])
@pytest.mark.parametrize("K,N", [(256, 64), (3584, 512), (18944, 64), (2048, 300)])
def test_kquant_matmul_matches_oracle(device, qt, K, N):
    rng = np.random.default_rng(K + N)
    w = oracle.synth_quantized(qt, 6, K, K * N)
    t = PackedTensor.upload(qt, w, K * N)
    x = rng.standard_normal(K).astype(np.float32)
    y = np.empty(N, np.float32)
    Linear.matmul(y, x, t, 0, K, N)
    assert rel(y, oracle.matvec(qt, w, 0, x, K, N)) < TOL


@pytest.mark.parametrize("qt", [C.TYPE_Q4_K, C.TYPE_Q6_K])
@pytest.mark.parametrize("batch", [2, 3, 8, 16, 21])
def test_kquant_matmul_batched(device, qt, batch):
    """The batched K-quant matvec (up to 16 vectors per launch, more in
    launch groups; 37 rows: a partial row group) against the oracle, vector
    by vector."""
    K, Nr = 3584, 37
    rng = np.random.default_rng(batch)
    w = oracle.synth_quantized(qt, 17, K, K * Nr)
    t = PackedTensor.upload(qt, w, K * Nr)
    x = rng.standard_normal((batch, K)).astype(np.float32)
    xd = torch.from_numpy(x).cuda()
    yd = torch.full((batch, Nr), float("nan"), dtype=torch.float32, device="cuda")
    Linear.matmul_device(yd.data_ptr(), xd.data_ptr(), t, 0, K, Nr, batch)
    torch.cuda.synchronize()
    y = yd.cpu().numpy()
    for b in range(batch):
        assert rel(y[b], oracle.matvec(qt, w, 0, x[b], K, Nr)) < TOL, b
    t.free()


def test_matmul_classifier_shape(device):
    K, N = 2048, 151936
    w = oracle.synth_quantized(C.TYPE_Q8_0, 8, 1, K * N)
    t = PackedTensor.upload(C.TYPE_Q8_0, w, K * N)
    x = np.random.default_rng(1).standard_normal(K).astype(np.float32)
    y = np.empty(N, np.float32)
    Linear.matmul(y, x, t, 0, K, N)
    ref = oracle.matvec(C.TYPE_Q8_0, w, 0, x, K, N)
    assert rel(y, ref) < TOL
    assert int(np.argmax(y)) == int(np.argmax(ref))


def test_matmul_weights_offset_layers(device):
    """weightsOffset = layer*in*out into a concatenated tensor (Linear.java:43-44)."""
    K, N, L = 576, 192, 3
    w = oracle.synth_quantized(C.TYPE_Q8_0, 9, 2, K * N * L)
    t = PackedTensor.upload(C.TYPE_Q8_0, w, K * N * L)
    x = np.random.default_rng(2).standard_normal(K).astype(np.float32)
    for layer in range(L):
        y = np.empty(N, np.float32)
        Linear.matmul(y, x, t, layer * K * N, K, N)
        assert rel(y, oracle.matvec(C.TYPE_Q8_0, w, layer * K * N, x, K, N)) < TOL


def test_matmul_errors(device):
    N = native
    K, rows = 64, 32
    t = PackedTensor.upload(C.TYPE_Q8_0, oracle.synth_quantized(C.TYPE_Q8_0, 1, 1, K * rows), K * rows)
    x = np.zeros(K, np.float32)
    y = np.zeros(rows + 1, np.float32)
    with pytest.raises(N.IllegalStateException):        # Linear.java:46-50
        Linear.matmul(y, x, t, 0, K, rows + 1)
    with pytest.raises(N.IllegalStateException):
        Linear.matmul(y, x, t, 32, K, rows)
    with pytest.raises(N.IllegalArgumentException):     # not whole blocks
        Linear.matmul(y, x, t, 0, 48, 8)
    with pytest.raises(N.IllegalArgumentException):
        Linear.matmul(y, None, t, 0, K, rows)
    Linear.matmul(y, x, t, 0, K, 0)                      # outputSize 0: no work


@pytest.mark.parametrize("qt", [C.TYPE_Q8_0, C.TYPE_Q4_0])
@pytest.mark.parametrize("batch", [2, 3, 8, 13, 32, 40])
def test_matmul_batched(device, qt, batch):
    K, N = 2048, 1000
    w = oracle.synth_quantized(qt, 10, batch, K * N)
    t = PackedTensor.upload(qt, w, K * N)
    X = torch.randn(batch, K, dtype=torch.float32, generator=torch.Generator().manual_seed(batch))
    xd = X.cuda()
    yd = torch.empty(batch, N, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    Linear.matmul_device(yd.data_ptr(), xd.data_ptr(), t, 0, K, N, batch)
    torch.cuda.synchronize()
    Y = yd.cpu().numpy()
    for b in range(batch):
        assert rel(Y[b], oracle.matvec(qt, w, 0, X[b].numpy(), K, N)) < TOL, b
