"""Pins the oracle's block formats and fp16 handling.

The reference has no tests or fixtures; the pins are gguf-py 0.19.0's own
quantize/dequantize outputs (tests/golden/block_formats.npz, made by
tests/golden/make_golden.py) and numpy's IEEE fp16 conversions.
"""
import os

import numpy as np
import pytest

import oracle
from brewference_b200.config import TYPE_Q4_0, TYPE_Q4_K, TYPE_Q6_K, TYPE_Q8_0

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "block_formats.npz")


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


@pytest.mark.parametrize("name,qt", [("q8_0", TYPE_Q8_0), ("q4_0", TYPE_Q4_0)])
def test_quantize_matches_gguf_py(golden, name, qt):
    q = oracle.quantize(qt, golden[f"{name}_x"])
    assert np.array_equal(q, golden[f"{name}_bytes"])


@pytest.mark.parametrize("name,qt", [("q8_0", TYPE_Q8_0), ("q4_0", TYPE_Q4_0), ("q4_k", TYPE_Q4_K), ("q6_k", TYPE_Q6_K)])
def test_dequantize_bit_exact_vs_gguf_py(golden, name, qt):
    ref = golden[f"{name}_deq"]
    d = oracle.dequantize(qt, golden[f"{name}_bytes"], 0, ref.size)
    assert np.array_equal(d.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("name,qt,be", [("q8_0", TYPE_Q8_0, 32), ("q4_k", TYPE_Q4_K, 256), ("q6_k", TYPE_Q6_K, 256)])
def test_dequantize_at_offsets(golden, name, qt, be):
    """dequantizeRow at an element offset (QuantizedWeights.java:76-85)."""
    ref = golden[f"{name}_deq"]
    for off, n in ((be, be), (3 * be, 2 * be), (5, 40)):
        d = oracle.dequantize(qt, golden[f"{name}_bytes"], off, n)
        assert np.array_equal(d.view(np.uint32), ref[off:off + n].view(np.uint32))


def test_half_to_float_exhaustive():
    """HalfPrecisionFloat.toFloat on all 65536 patterns vs IEEE widening."""
    h = np.arange(65536, dtype=np.uint16)
    ref = h.view(np.float16).astype(np.float32)
    mine = np.array([oracle.half_to_float(int(v)) for v in h], np.float32)
    nan = np.isnan(ref)
    assert np.array_equal(mine.view(np.uint32)[~nan], ref.view(np.uint32)[~nan])
    assert np.isnan(mine[nan]).all()


def test_float_to_half_rne():
    rng = np.random.default_rng(3)
    f = (rng.standard_normal(20000) * np.exp2(rng.integers(-30, 18, 20000))).astype(np.float32)
    edge = np.array([65504, 65519.99, 65520, 1e-8, 2.98e-8, 2.9802322e-8, 5.96e-8, 6.1e-5, 0.0, -0.0, np.inf, -np.inf],
                    np.float32)
    f = np.concatenate([f, edge])
    mine = np.array([oracle.float_to_half(float(v)) for v in f], np.uint16)
    with np.errstate(over="ignore"):
        ref = f.astype(np.float16).view(np.uint16)
    assert np.array_equal(mine, ref)


def test_synth_values_deterministic_and_normal():
    a = oracle.synth_fill(7, 0x30001, 0, 200000, 0.02)
    b = oracle.synth_fill(7, 0x30001, 0, 200000, 0.02)
    assert np.array_equal(a, b)
    assert abs(a.mean()) < 2e-4 and abs(a.std() - 0.02) < 2e-4
    c = oracle.synth_fill(7, 0x30002, 0, 1000, 0.02)
    assert not np.array_equal(a[:1000], c)
    # offset windows are consistent
    assert np.array_equal(oracle.synth_fill(7, 0x30001, 100, 50, 0.02), a[100:150])


@pytest.mark.parametrize("qt", [TYPE_Q8_0, TYPE_Q4_0, TYPE_Q4_K, TYPE_Q6_K])
def test_synth_quantized_roundtrip_error(qt):
    n = 256 * 64
    q = oracle.synth_quantized(qt, 11, 5, n)
    x = oracle.synth_fill(11, 5, 0, n, 0.02)
    d = oracle.dequantize(qt, q, 0, n)
    rel = np.linalg.norm(d - x) / np.linalg.norm(x)
    bound = {TYPE_Q8_0: 0.01, TYPE_Q4_0: 0.12, TYPE_Q4_K: 0.12, TYPE_Q6_K: 0.04}[qt]
    assert rel < bound, rel
