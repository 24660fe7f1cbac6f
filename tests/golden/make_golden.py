"""Generates the golden block-format fixtures with gguf-py 0.19.0.

gguf-py (the `gguf` package, gguf/quants.py) is GGML's own Python
implementation of the block formats.  The reference decodes only Q8_0 and
has no tests or fixtures, so these vectors pin the oracle's (and through it
the CUDA path's) quantize/dequantize arithmetic:

  q8_0 / q4_0 : float32 input -> gguf.quants.quantize bytes -> dequantize
  q4_k / q6_k : random valid blocks (finite fp16 scales) -> dequantize
                (gguf-py has no quantizer for the K-quants)

Run from the repository root:  python tests/golden/make_golden.py
"""
import os

import numpy as np
import gguf
from gguf import GGMLQuantizationType as T
from gguf.quants import dequantize, quantize

HERE = os.path.dirname(os.path.abspath(__file__))


def finite_half_bytes(rng, n, lo_exp=-14, hi_exp=-4):
    """random fp16 values of both signs with exponents in [lo_exp, hi_exp]"""
    mant = rng.uniform(1.0, 2.0, n)
    ex = rng.integers(lo_exp, hi_exp + 1, n)
    sign = rng.choice([-1.0, 1.0], n)
    return (sign * mant * np.exp2(ex)).astype(np.float16).view(np.uint8).reshape(n, 2)


def main():
    rng = np.random.default_rng(20261201)
    out = {}
    # Q8_0 / Q4_0: 96 blocks of N(0, 0.02) plus edge blocks
    x = (rng.standard_normal(96 * 32) * 0.02).astype(np.float32)
    edge = np.zeros((6, 32), np.float32)
    edge[1] = 1.0                                   # all equal
    edge[2] = np.linspace(-1, 1, 32)                 # symmetric ramp
    edge[3, 7] = -3.5                                # single negative peak
    edge[4] = rng.standard_normal(32) * 1e-6         # tiny values: subnormal fp16 scales
    edge[5] = rng.standard_normal(32) * 300.0        # large values
    x = np.concatenate([x, edge.ravel()]).astype(np.float32)
    for name, qt in (("q8_0", T.Q8_0), ("q4_0", T.Q4_0)):
        q = quantize(x.reshape(-1, 32), qt).reshape(-1)
        out[f"{name}_x"] = x
        out[f"{name}_bytes"] = q
        out[f"{name}_deq"] = dequantize(q, qt).reshape(-1).astype(np.float32)
    # Q4_K: 24 random blocks of 144 bytes
    nb = 24
    b = rng.integers(0, 256, (nb, 144), dtype=np.uint8)
    b[:, 0:2] = finite_half_bytes(rng, nb, -14, -6)
    b[:, 2:4] = finite_half_bytes(rng, nb, -14, -6)
    b[:, 0:2][: 2] = np.array([0, 0], np.uint8)      # zero d in two blocks
    out["q4_k_bytes"] = b.reshape(-1)
    out["q4_k_deq"] = dequantize(b.reshape(-1), T.Q4_K).reshape(-1).astype(np.float32)
    # Q6_K: 24 random blocks of 210 bytes
    b = rng.integers(0, 256, (nb, 210), dtype=np.uint8)
    b[:, 208:210] = finite_half_bytes(rng, nb, -14, -6)
    out["q6_k_bytes"] = b.reshape(-1)
    out["q6_k_deq"] = dequantize(b.reshape(-1), T.Q6_K).reshape(-1).astype(np.float32)
    out["gguf_version"] = np.array(getattr(gguf, "__version__", "0.19.0"))
    np.savez_compressed(os.path.join(HERE, "block_formats.npz"), **out)
    print("wrote", os.path.join(HERE, "block_formats.npz"))


if __name__ == "__main__":
    main()
