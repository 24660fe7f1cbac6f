"""The integer identities the tcgen05 K-quant matvec (csrc/kqtc.cu) rests on,
checked on the CPU: every Q4_K / Q6_K element's integer factor, with its
sub-block scale folded in, splits exactly into two int8 limbs; every
integer sum of a 256-element super-block stays below 2^22 in magnitude (so
tensor-memory cells preset to the bits of 1.5 * 2^23 read back exact); and,
on blocks quantized by the oracle, the expanded form computes the same dot
product as the oracle's dequantized rows, also with the Q4_K min term taken
from fp32 sub-block sums as the matvec's epilogue forms it."""
import numpy as np
import pytest

import oracle
from brewference_b200.config import TYPE_Q4_K, TYPE_Q6_K

MAGIC_RANGE = 1 << 22
LIMB_MAX = 128   # |hi|, |mid|, |lo| of the 24-bit activation split


def test_q4k_scale_split_exhaustive():
    sc = np.arange(64)[:, None]
    q = np.arange(16)[None, :]
    h, l = q * (sc >> 3), q * (sc & 7)
    assert np.array_equal(8 * h + l, sc * q)
    assert h.min() >= 0 and l.min() >= 0 and max(h.max(), l.max()) <= 105   # int8, non-negative
    assert 256 * 105 * LIMB_MAX < MAGIC_RANGE                                # a super-block's h or l sum


def test_q6k_scale_split_exhaustive():
    sc = np.arange(-128, 128)[:, None]
    qq = np.arange(-32, 32)[None, :]
    v = sc * qq
    h, l = v >> 6, v & 63
    assert np.array_equal(64 * h + l, v)
    assert h.min() >= -64 and h.max() <= 64 and l.min() >= 0 and l.max() <= 63
    assert 256 * 64 * LIMB_MAX < MAGIC_RANGE and 256 * 63 * LIMB_MAX < MAGIC_RANGE


def _half(b, o):
    """The little-endian fp16 at byte o of block b (an array of byte values)."""
    return float(np.array([int(b[o]) | (int(b[o + 1]) << 8)], dtype=np.uint16).view(np.float16)[0])


def _q4k_fields(blk):
    """d, dmin, per sub-block (sc, m) and the 256 quants of one Q4_K block
    (GGML's layout; get_scale_min_k4)."""
    s = blk[4:16]
    sc, m = [], []
    for j in range(8):
        if j < 4:
            sc.append(s[j] & 63)
            m.append(s[j + 4] & 63)
        else:
            sc.append((s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4))
            m.append((s[j + 4] >> 4) | ((s[j] >> 6) << 4))
    q = np.array([(blk[16 + 32 * (j // 2) + k] >> (4 * (j & 1))) & 15 for j in range(8) for k in range(32)])
    return _half(blk, 0), _half(blk, 2), np.array(sc), np.array(m), q


def _q6k_fields(blk):
    """d, the 16 int8 scales and the 256 quants q - 32 of one Q6_K block."""
    q = []
    for r in range(256):
        hb, rr = r // 128, r % 128
        grp, ll = rr // 32, rr % 32
        lq = blk[64 * hb + (grp & 1) * 32 + ll]
        low = (lq & 15) if grp < 2 else (lq >> 4)
        high = (blk[128 + 32 * hb + ll] >> (2 * grp)) & 3
        q.append((low | (high << 4)) - 32)
    return _half(blk, 208), blk[192:208].astype(np.int8).astype(np.int64), np.array(q)


def _limbs(x):
    """The 24-bit three-limb split of one super-block of x (prep.cuh)."""
    am = np.abs(x).max()
    v = np.rint(x.astype(np.float64) * (8290000.0 / am)).astype(np.int64)
    lo = ((v + 128) & 255) - 128
    v1 = (v - lo) >> 8
    mid = ((v1 + 128) & 255) - 128
    hi = (v1 - mid) >> 8
    assert np.abs(np.stack([hi, mid, lo])).max() <= LIMB_MAX
    return am / 8290000.0, (hi, mid, lo)


@pytest.mark.parametrize("qt", [TYPE_Q4_K, TYPE_Q6_K])
def test_expanded_superblock_dot_matches_oracle(qt):
    """Per super-block: s * sum_limbs 2^{16,8,0} * (d (F h.limb + l.limb) -
    dmin sum_j m_j X_j), with every inner sum an exact integer, equals the
    oracle's dequantized row times x up to fp32 rounding of the factors."""
    rng = np.random.default_rng(11 + qt)
    K = 1024
    w = oracle.quantize(qt, (rng.standard_normal(K) * 0.02).astype(np.float32))
    x = rng.standard_normal(K).astype(np.float32)
    ref = float(oracle.dequantize(qt, w, 0, K).astype(np.float64) @ x.astype(np.float64))
    bb = 144 if qt == TYPE_Q4_K else 210
    total = 0.0
    for sb in range(K // 256):
        blk = np.frombuffer(bytes(w[sb * bb:(sb + 1) * bb]), dtype=np.uint8).astype(np.int64)
        s, limbs = _limbs(x[sb * 256:(sb + 1) * 256])
        if qt == TYPE_Q4_K:
            d, dmin, sc, m, q = _q4k_fields(blk)
            scl = np.repeat(sc, 32)
            h, l, F = q * (scl >> 3), q * (scl & 7), 8
        else:
            d, sc, q = _q6k_fields(blk)
            v = np.repeat(sc, 16) * q
            h, l, F, dmin, m = v >> 6, v & 63, 64, 0.0, np.zeros(8, np.int64)
        acc = 0.0
        for weight, lim in zip((65536.0, 256.0, 1.0), limbs):
            hs, ls = int(h @ lim), int(l @ lim)
            msum = int(m @ lim.reshape(8, 32).sum(axis=1))
            assert max(abs(hs), abs(ls), abs(msum)) < MAGIC_RANGE
            acc += weight * (d * (F * hs + ls) - dmin * msum)
        total += s * acc
    # tolerance: 1e-7 of sum |w x| (the fp32 factors d, dmin and the x scale
    # are the only rounded quantities)
    assert abs(total - ref) <= 1e-7 * np.abs(oracle.dequantize(qt, w, 0, K)).astype(np.float64) @ np.abs(x)


def test_q4k_min_term_from_fp32_subblock_sums():
    """The Q4_K min term as the matvec computes it now: the records carry,
    per vector and sub-block, the exact integer 2^16 sum(hi) + 2^8 sum(mid)
    + sum(lo) (an int32: |.| < 2^28) rounded once to fp32 and scaled by s;
    the epilogue forms -dmin sum_j m_j X_j with fp32 FMAs beside the integer
    h / l sums.  Against the oracle's dequantized row times x."""
    rng = np.random.default_rng(29)
    K = 2048
    f32 = np.float32
    for trial in range(4):
        w = oracle.quantize(TYPE_Q4_K, (rng.standard_normal(K) * 0.02).astype(np.float32))
        x = (rng.standard_normal(K) * (1.0 + 10.0 * trial)).astype(np.float32)
        ref = float(oracle.dequantize(TYPE_Q4_K, w, 0, K).astype(np.float64) @ x.astype(np.float64))
        total = 0.0
        for sb in range(K // 256):
            blk = np.frombuffer(bytes(w[sb * 144:(sb + 1) * 144]), dtype=np.uint8).astype(np.int64)
            s, (hi, mid, lo) = _limbs(x[sb * 256:(sb + 1) * 256])
            d, dmin, sc, m, q = _q4k_fields(blk)
            scl = np.repeat(sc, 32)
            h, l = q * (scl >> 3), q * (scl & 7)
            main = 0.0
            for weight, lim in zip((65536.0, 256.0, 1.0), (hi, mid, lo)):
                main += weight * (d * (8 * int(h @ lim) + int(l @ lim)))
            st = (65536 * hi.reshape(8, 32).sum(axis=1) + 256 * mid.reshape(8, 32).sum(axis=1)
                  + lo.reshape(8, 32).sum(axis=1))
            assert np.abs(st).max() < 2 ** 28
            X = st.astype(f32) * f32(s)                      # one rounding, then the scale
            mx = f32(0.0)
            for j in range(8):                               # fp32 FMAs in sub-block order
                mx = f32(np.float64(f32(m[j])) * np.float64(X[j]) + np.float64(mx))
            total += s * main - dmin * float(mx)
        tol = 2e-7 * float(np.abs(oracle.dequantize(TYPE_Q4_K, w, 0, K)).astype(np.float64) @ np.abs(x))
        assert abs(total - ref) <= tol, (trial, abs(total - ref), tol)
