"""Whole-model parity of the unfused forward used by models with K-quant
matrices (Q4_K / Q6_K, the Qwen2.5-7B config's formats) against the
oracle's forward on the same seeded weights: logits within 1e-4 relative L2
at every checked step and the greedy tokens identical.  The K-quant rows
are dequantized with GGML's formulas (bit-exact dequant is checked in
test_gpu_matvec.py) and summed in fp32 in a different order than the
oracle's sequential sums, hence the tolerance.
"""
import numpy as np
import pytest

import oracle
from brewference_b200 import config as C
from brewference_b200.api import DeviceModel

pytestmark = pytest.mark.gpu
LOGIT_TOL = 1e-4
Q4K, Q6K, Q8, Q4 = C.TYPE_Q4_K, C.TYPE_Q6_K, C.TYPE_Q8_0, C.TYPE_Q4_0


def rel(a, b):
    return float(np.linalg.norm(a.astype(np.float64) - b) / np.linalg.norm(b.astype(np.float64)))


def kquant(cfg, embed=Q4K, out=Q6K, attn=Q4K, ffn=Q4K, down=Q6K, **kw):
    return cfg.replace(type_embed=embed, type_output=out, type_q=attn, type_k=attn, type_v=attn, type_o=attn,
                       type_gate=ffn, type_up=ffn, type_down=down, **kw)


def parity(cfg, seed, prompt_len, n_gen, check_steps=3):
    dm = DeviceModel.synthesize(cfg, seed)
    om = oracle.OracleModel(cfg, seed)
    rng = np.random.default_rng(seed)
    prompt = rng.integers(0, cfg.vocab_size, prompt_len).tolist()
    dm.reset()
    om.reset()
    for i in range(check_steps):
        lg, am = dm.forward([prompt[i]], [i])
        ref = om.forward(prompt[i], i)
        assert rel(lg[0], ref) < LOGIT_TOL, (i, rel(lg[0], ref))
        assert am[0] == int(np.argmax(lg[0]))
    got = dm.generate(prompt, n_gen)
    want = om.generate(prompt, n_gen)
    assert got == want
    dm.close()
    om.close()
    return got


SMALL = dict(n_layers=3, vocab_size=4096, seq_len=256)


def test_qwen2_kquant_small(device):
    """Qwen2 (QKV bias) with the 7B config's formats: Q4_K attention / FFN /
    embedding, Q6_K down and untied classifier."""
    cfg = kquant(C.qwen25_7b(), dim=1024, hidden_dim=2048, n_heads=8, n_kv_heads=4, **SMALL)
    parity(cfg, 71, prompt_len=16, n_gen=64)


@pytest.mark.parametrize("arch", [C.ARCH_LLAMA, C.ARCH_QWEN3, C.ARCH_GEMMA3, C.ARCH_GEMMA2, C.ARCH_SMOLLM3])
def test_other_archs_kquant(device, arch):
    kw = dict(SMALL)
    if arch == C.ARCH_LLAMA:
        base = C.smollm2_135m().replace(dim=512, hidden_dim=1536, n_heads=8, n_kv_heads=4, head_size=64)
    elif arch == C.ARCH_QWEN3:
        base = C.qwen3_1_7b().replace(dim=1024, hidden_dim=2048, n_heads=8, n_kv_heads=4)
    elif arch == C.ARCH_GEMMA2:
        base = C.gemma2_2b().replace(dim=1024, hidden_dim=2048, n_heads=4, n_kv_heads=2, sliding_window=8)
    elif arch == C.ARCH_SMOLLM3:   # layer 3 runs without RoPE
        base = C.smollm3_3b().replace(dim=1024, hidden_dim=2048, n_heads=8, n_kv_heads=4)
        kw["n_layers"] = 5
    else:
        base = C.gemma3_1b().replace(dim=1024, hidden_dim=2048, sliding_window=8)
    cfg = kquant(base, tied_embeddings=0, **kw)
    parity(cfg, 80 + arch, prompt_len=12, n_gen=48)


def test_mixed_types(device):
    """Q8_0 attention and Q4_0 gate/up beside Q4_K / Q6_K matrices in one model."""
    cfg = kquant(C.qwen25_7b(), dim=1024, hidden_dim=2048, n_heads=8, n_kv_heads=4, attn=Q8, ffn=Q4, **SMALL)
    parity(cfg, 93, prompt_len=10, n_gen=32)


def test_qwen25_7b_width_two_layers(device):
    """The 7B config's widths (3584 / 18944, 28 heads, 4 kv heads) with two
    layers and a reduced vocabulary."""
    cfg = C.qwen25_7b().replace(n_layers=2, vocab_size=8192, seq_len=128)
    parity(cfg, 7, prompt_len=6, n_gen=16, check_steps=2)


@pytest.mark.parametrize("B", [5, 20, 32])
def test_kquant_many_sequences(device, B):
    """Concurrent sequences up to 32 (the 7B config's workload size; the
    K-quant matvec takes up to 32 vectors per launch in one or two groups of
    16 MMA vectors, 5 and 20 leaving padded columns): a sequence's logits in
    the batch equal those of the same sequence forwarded alone, and
    sequence 0 matches the oracle."""
    cfg = kquant(C.qwen25_7b(), dim=1024, hidden_dim=2048, n_heads=8, n_kv_heads=4, **SMALL)
    steps = 3
    dm = DeviceModel.synthesize(cfg, 91, max_batch=B)
    toks = np.random.default_rng(5).integers(0, cfg.vocab_size, (steps, B)).astype(np.int32)
    batched = []
    for pos in range(steps):
        lg, am = dm.forward(toks[pos], np.full(B, pos, np.int32))
        assert all(am[b] == int(np.argmax(lg[b])) for b in range(B))
        batched.append(lg)
    dm.close()
    single = DeviceModel.synthesize(cfg, 91)
    for b in sorted({0, B // 2 + 1, B - 1}):
        single.reset()
        for pos in range(steps):
            lg, _ = single.forward([toks[pos][b]], [pos])
            assert rel(batched[pos][b], lg[0]) < 1e-6, (b, pos)
    single.close()
    om = oracle.OracleModel(cfg, 91)
    om.reset()
    for pos in range(steps):
        ref = om.forward(int(toks[pos][0]), pos)
        assert rel(batched[pos][0], ref) < LOGIT_TOL, (pos, rel(batched[pos][0], ref))
    om.close()
