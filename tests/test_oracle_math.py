"""The oracle's restatement of the Java arithmetic, checked on small cases
against straight-line Python written from the same Java lines."""
import math

import numpy as np
import pytest

import oracle
from brewference_b200 import config as C


def f32(v):
    return float(np.float32(v))


def java_matvec_q8(w_bytes, x, K, N):
    """Linear.computeRowDotProduct (Linear.java:76-99), pure Python, fp32 rounding per op."""
    out = []
    nb = K // 32
    for r in range(N):
        row_sum = np.float32(0)
        for b in range(nb):
            blk = w_bytes[(r * nb + b) * 34:(r * nb + b + 1) * 34]
            scale = np.frombuffer(bytes(blk[:2]), np.float16)[0].astype(np.float32)
            q = np.frombuffer(bytes(blk[2:]), np.int8)
            bs = np.float32(0)
            for i in range(32):
                bs = np.float32(bs + np.float32(np.float32(q[i]) * x[b * 32 + i]))
            row_sum = np.float32(row_sum + np.float32(bs * scale))
        out.append(row_sum)
    return np.array(out, np.float32)


def test_matvec_q8_0_bit_exact_vs_java_order():
    rng = np.random.default_rng(0)
    K, N = 96, 7
    w = oracle.quantize(C.TYPE_Q8_0, (rng.standard_normal(K * N) * 0.02).astype(np.float32))
    x = rng.standard_normal(K).astype(np.float32)
    y = oracle.matvec(C.TYPE_Q8_0, w, 0, x, K, N)
    ref = java_matvec_q8(w, x, K, N)
    assert np.array_equal(y.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("qt", [C.TYPE_Q8_0, C.TYPE_Q4_0, C.TYPE_Q4_K, C.TYPE_Q6_K])
def test_matvec_close_to_float64(qt):
    rng = np.random.default_rng(1)
    K, N = 512, 300   # N >= 256: the row-parallel path
    w = oracle.synth_quantized(qt, 3, 9, K * N)
    x = rng.standard_normal(K).astype(np.float32)
    y = oracle.matvec(qt, w, 0, x, K, N)
    W = oracle.dequantize(qt, w, 0, K * N).reshape(N, K).astype(np.float64)
    ref = W @ x.astype(np.float64)
    assert np.linalg.norm(y - ref) / np.linalg.norm(ref) < 1e-5


def test_matvec_weights_offset():
    rng = np.random.default_rng(2)
    K, N, L = 64, 32, 3
    w = oracle.synth_quantized(C.TYPE_Q8_0, 4, 1, K * N * L)
    x = rng.standard_normal(K).astype(np.float32)
    for layer in range(L):
        y = oracle.matvec(C.TYPE_Q8_0, w, layer * K * N, x, K, N)
        seg = w[layer * K * N // 32 * 34:(layer + 1) * K * N // 32 * 34]
        assert np.array_equal(y, oracle.matvec(C.TYPE_Q8_0, seg, 0, x, K, N))


def test_rmsnorm_java_formula():
    rng = np.random.default_rng(4)
    x = rng.standard_normal(64).astype(np.float32)
    w = rng.standard_normal(64).astype(np.float32)
    ss = np.float32(0)
    for v in x:
        ss = np.float32(ss + np.float32(v * v))
    ms = np.float32(ss / np.float32(64))
    scale = np.float32(1.0 / math.sqrt(float(np.float32(ms + np.float32(1e-5)))))
    ref = np.array([np.float32(np.float32(x[i] * scale) * w[i]) for i in range(64)], np.float32)
    assert np.array_equal(oracle.rmsnorm(x, w, 1e-5), ref)


def test_softmax_and_argmax():
    v = np.array([1.0, 3.0, 3.0, -2.0], np.float32)
    s = oracle.softmax(v)
    assert abs(s.sum() - 1) < 1e-6 and s[1] == s[2]
    assert oracle.argmax(v) == 1            # first maximum (Kernels.java:150-162)
    assert oracle.argmax(np.array([-1.0, -1.0], np.float32)) == 0


@pytest.mark.parametrize("interleaved", [True, False])
def test_rope_matches_java(interleaved):
    rng = np.random.default_rng(5)
    hs, nh, nkv, pos, base = 8, 2, 1, 17.0, 10000.0
    q = rng.standard_normal(nh * hs).astype(np.float32)
    k = rng.standard_normal(nkv * hs).astype(np.float32)
    qo, ko = oracle.rope(q, k, nh, nkv, hs, base, pos, interleaved)
    half = hs // 2
    cs, sn = [], []
    for p in range(half):
        invf = f32(1.0 / math.pow(base, f32(f32(2 * p) / f32(hs))))
        ang = f32(np.float32(pos) * np.float32(invf))
        cs.append(np.float32(math.cos(ang)))
        sn.append(np.float32(math.sin(ang)))
    def apply(v, heads):
        v = v.copy()
        for h in range(heads):
            for d in range(half):
                i0 = h * hs + (2 * d if interleaved else d)
                i1 = h * hs + (2 * d + 1 if interleaved else d + half)
                a, b = v[i0], v[i1]
                v[i0] = np.float32(np.float32(a * cs[d]) - np.float32(b * sn[d]))
                v[i1] = np.float32(np.float32(a * sn[d]) + np.float32(b * cs[d]))
        return v
    assert np.array_equal(qo, apply(q, nh)) and np.array_equal(ko, apply(k, nkv))


@pytest.mark.parametrize("gelu", [False, True])
def test_glu(gelu):
    rng = np.random.default_rng(6)
    hb = rng.standard_normal(33).astype(np.float32)
    hb2 = rng.standard_normal(33).astype(np.float32)
    out = oracle.glu(hb, hb2, gelu)
    ref = []
    for a, b in zip(hb, hb2):
        v = float(a)
        if gelu:
            inner = float(np.float32(0.7978845608028654)) * (v + float(np.float32(0.044715)) * v * v * v)
            act = 0.5 * v * (1.0 + math.tanh(inner))
        else:
            act = v / (1.0 + math.exp(-v))
        ref.append(np.float32(np.float32(act) * b))
    assert np.array_equal(out, np.array(ref, np.float32))


def tiny(arch):
    base = {C.ARCH_LLAMA: C.smollm2_135m, C.ARCH_QWEN3: C.qwen3_1_7b, C.ARCH_GEMMA3: C.gemma3_1b,
            C.ARCH_QWEN2: C.qwen25_7b}[arch]()
    return base.replace(n_layers=2, vocab_size=512, seq_len=64, dim=256 if arch != C.ARCH_GEMMA3 else 256,
                        hidden_dim=512, n_heads=4, n_kv_heads=2, head_size=64, sliding_window=8)


@pytest.mark.parametrize("arch", [C.ARCH_LLAMA, C.ARCH_QWEN2, C.ARCH_QWEN3, C.ARCH_GEMMA3])
def test_generate_token_feeding_order(arch):
    """GenericModelSession: prefill forwards prompt[i] at i, then the last
    prompt token again at n_prompt, then each argmax at the next position
    (runtime/ModelRunner.java:141-152,196-206)."""
    cfg = tiny(arch)
    m = oracle.OracleModel(cfg, 99)
    prompt = [3, 7, 11, 5]
    gen = m.generate(prompt, 6)
    m.reset()
    for i, t in enumerate(prompt):
        m.forward(t, i)
    pending, pos, manual = prompt[-1], len(prompt), []
    for _ in range(6):
        tok = int(np.argmax(m.forward(pending, pos)))
        manual.append(tok)
        pending, pos = tok, pos + 1
    assert gen == manual


def test_generate_limits_and_eos():
    cfg = tiny(C.ARCH_LLAMA)
    m = oracle.OracleModel(cfg, 5)
    full = m.generate([1, 2], 5)
    eos_cfg = cfg.replace(eos_token=full[2])
    m2 = oracle.OracleModel(eos_cfg, 5)
    stop = m2.generate([1, 2], 5)
    assert stop == full[: full.index(full[2]) + 1]            # EOS included, then stop
    assert len(m.generate([1] * 60, 0)) == cfg.seq_len - 60    # max_new <= 0: rest of the context
    with pytest.raises(RuntimeError):
        m.generate([1] * (cfg.seq_len + 1), 1)                 # ensureContextAvailable
