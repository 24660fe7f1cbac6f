"""The batched prefill (brew_model_set_prefill(BATCHED): prompt chunks through
each layer together, matrices on the tcgen05 GEMM) against the token-by-token
prefill and the oracle.  The state a prefill leaves is the KV cache; it is
checked through the logits of the next position (which read every cache row
of every layer): within 1e-4 relative L2 of the oracle's logits (the
oracle's forward fed the prompt token by token, as the reference's
ModelRunner.prefill does), and the greedy tokens generated afterwards equal
to those after the token-by-token prefill."""
import numpy as np
import pytest

import oracle
from brewference_b200 import _native as N
from brewference_b200 import config as C
from brewference_b200.api import PREFILL_BATCHED, PREFILL_TOKENS, DeviceModel

pytestmark = pytest.mark.gpu
LOGIT_TOL = 1e-4
Q8 = dict(type_embed=C.TYPE_Q8_0, type_output=C.TYPE_Q8_0, type_q=C.TYPE_Q8_0, type_k=C.TYPE_Q8_0,
          type_v=C.TYPE_Q8_0, type_o=C.TYPE_Q8_0, type_gate=C.TYPE_Q8_0, type_up=C.TYPE_Q8_0, type_down=C.TYPE_Q8_0)


def rel(a, b):
    return float(np.linalg.norm(a.astype(np.float64) - b) / np.linalg.norm(b.astype(np.float64)))


def small(arch, **kw):
    """Small models of each architecture whose matrix row counts are
    multiples of 128 (the GEMM's tile)."""
    kw.setdefault("n_layers", 3)
    kw.setdefault("vocab_size", 4096)
    kw.setdefault("seq_len", 256)
    kw.update(Q8)
    if arch == C.ARCH_LLAMA:     # interleaved RoPE, head size 64
        return C.smollm2_135m().replace(dim=512, hidden_dim=1024, n_heads=8, n_kv_heads=4, **kw)
    if arch == C.ARCH_QWEN2:     # QKV bias
        return C.qwen25_7b().replace(dim=1024, hidden_dim=2048, n_heads=8, n_kv_heads=4, tied_embeddings=1, **kw)
    if arch == C.ARCH_QWEN3:     # QK-norm
        return C.qwen3_1_7b().replace(dim=512, hidden_dim=1536, n_heads=8, n_kv_heads=4, **kw)
    if arch == C.ARCH_SMOLLM3:   # interleaved RoPE, none on layer 3
        kw["n_layers"] = 5
        return C.smollm3_3b().replace(dim=1024, hidden_dim=2048, n_heads=8, n_kv_heads=4, **kw)
    kw.setdefault("sliding_window", 16)   # Gemma: head size 256, local / global layers, post-norms, GeGLU
    if arch == C.ARCH_GEMMA2:    # no QK-norm, global every 2nd layer
        return C.gemma2_2b().replace(dim=1024, hidden_dim=2048, n_heads=4, n_kv_heads=2, **kw)
    return C.gemma3_1b().replace(dim=1152, hidden_dim=2304, **kw)


def next_logits(dm, prompt, mode):
    """Prefill in `mode`, then the logits of the last prompt token at the next
    position (the first step of generate)."""
    dm.set_prefill(mode)
    dm.prefill(prompt)
    lg, am = dm.forward([prompt[-1]], [len(prompt)])
    return lg[0]


def oracle_logits(cfg, seed, prompt):
    om = oracle.OracleModel(cfg, seed)
    om.reset()
    for i, t in enumerate(prompt):
        om.forward(t, i)
    out = om.forward(prompt[-1], len(prompt))
    om.close()
    return out


@pytest.mark.parametrize("arch", [C.ARCH_LLAMA, C.ARCH_QWEN2, C.ARCH_QWEN3, C.ARCH_GEMMA3, C.ARCH_GEMMA2, C.ARCH_SMOLLM3])
def test_batched_prefill_matches_oracle_and_tokens(device, arch):
    cfg = small(arch, n_layers=3 if arch != C.ARCH_GEMMA3 else 7)
    seed = 2000 + arch
    prompt = np.random.default_rng(seed).integers(0, cfg.vocab_size, 45).tolist()   # not a multiple of 32
    dm = DeviceModel.synthesize(cfg, seed)
    ref = oracle_logits(cfg, seed, prompt)
    lt = next_logits(dm, prompt, PREFILL_TOKENS)
    lb = next_logits(dm, prompt, PREFILL_BATCHED)
    assert rel(lt, ref) < LOGIT_TOL, rel(lt, ref)
    assert rel(lb, ref) < LOGIT_TOL, rel(lb, ref)
    # greedy tokens after each prefill
    dm.set_prefill(PREFILL_TOKENS)
    gt = dm.generate(prompt, 24)
    dm.set_prefill(PREFILL_BATCHED)
    gb = dm.generate(prompt, 24)
    assert gt == gb
    dm.close()


def test_batched_prefill_chunks(device):
    """A 700-token prompt: two chunks (512 + 188), the second attending to the
    first chunk's cache rows."""
    cfg = small(C.ARCH_QWEN3, n_layers=2, seq_len=1024)
    seed = 31
    prompt = np.random.default_rng(seed).integers(0, cfg.vocab_size, 700).tolist()
    dm = DeviceModel.synthesize(cfg, seed)
    ref = oracle_logits(cfg, seed, prompt)
    lb = next_logits(dm, prompt, PREFILL_BATCHED)
    lt = next_logits(dm, prompt, PREFILL_TOKENS)
    assert rel(lb, ref) < LOGIT_TOL, rel(lb, ref)
    assert rel(lt, ref) < LOGIT_TOL, rel(lt, ref)
    dm.set_prefill(PREFILL_BATCHED)
    dm.prefill(prompt)
    gb = dm.decode(16)
    dm.set_prefill(PREFILL_TOKENS)
    dm.prefill(prompt)
    gt = dm.decode(16)
    assert gb == gt
    dm.close()


Q4_LAYERS = dict(type_q=C.TYPE_Q4_0, type_k=C.TYPE_Q4_0, type_v=C.TYPE_Q4_0, type_o=C.TYPE_Q4_0,
                 type_gate=C.TYPE_Q4_0, type_up=C.TYPE_Q4_0, type_down=C.TYPE_Q4_0)


@pytest.mark.parametrize("arch", [C.ARCH_QWEN3, C.ARCH_GEMMA3])
def test_batched_prefill_q4_0_layers(device, arch):
    """Q4_0 layer matrices (the Gemma-3-1B config's format): the GEMM takes
    their quants as q - 8 with the same fp16 scales."""
    cfg = small(arch, n_layers=3 if arch != C.ARCH_GEMMA3 else 7).replace(**Q4_LAYERS)
    seed = 3100 + arch
    prompt = np.random.default_rng(seed).integers(0, cfg.vocab_size, 70).tolist()
    dm = DeviceModel.synthesize(cfg, seed)
    ref = oracle_logits(cfg, seed, prompt)
    lb = next_logits(dm, prompt, PREFILL_BATCHED)
    assert rel(lb, ref) < LOGIT_TOL, rel(lb, ref)
    dm.set_prefill(PREFILL_TOKENS)
    gt = dm.generate(prompt, 16)
    dm.set_prefill(PREFILL_BATCHED)
    gb = dm.generate(prompt, 16)
    assert gt == gb
    dm.close()


def test_batched_prefill_unsupported(device):
    # K-quant layers: no GEMM layout for them
    cfg = small(C.ARCH_QWEN3).replace(type_q=C.TYPE_Q4_K, type_k=C.TYPE_Q4_K, type_v=C.TYPE_Q4_K,
                                      type_o=C.TYPE_Q4_K, type_gate=C.TYPE_Q4_K, type_up=C.TYPE_Q4_K,
                                      type_down=C.TYPE_Q6_K)
    dm = DeviceModel.synthesize(cfg, 5)
    with pytest.raises(N.BrewError) as e:
        dm.set_prefill(PREFILL_BATCHED)
    assert e.value.code == N.ERR_UNSUPPORTED
    with pytest.raises(N.IllegalArgumentException):
        dm.set_prefill(7)
    dm.set_prefill(PREFILL_TOKENS)   # the default stays available
    dm.close()


@pytest.mark.parametrize("n", [1, 32, 512, 513])
def test_batched_prefill_lengths(device, n):
    """Prompt lengths at the edges of the token tile (32) and of a chunk
    (512; 513 leaves a 1-token second chunk)."""
    cfg = small(C.ARCH_QWEN3, n_layers=2, seq_len=640)
    seed = 40 + n
    prompt = np.random.default_rng(seed).integers(0, cfg.vocab_size, n).tolist()
    dm = DeviceModel.synthesize(cfg, seed)
    lb = next_logits(dm, prompt, PREFILL_BATCHED)
    lt = next_logits(dm, prompt, PREFILL_TOKENS)
    assert rel(lb, lt) < LOGIT_TOL, rel(lb, lt)
    dm.close()


def test_batched_prefill_context_full(device):
    """A prompt longer than the context is refused before any work, as in
    the token-by-token prefill (ModelRunner.java:208-216)."""
    cfg = small(C.ARCH_QWEN3, n_layers=1, seq_len=64)
    dm = DeviceModel.synthesize(cfg, 3)
    dm.set_prefill(PREFILL_BATCHED)
    with pytest.raises(N.BrewError) as e:
        dm.prefill(list(range(65)))
    assert e.value.code == N.ERR_CONTEXT_FULL
    dm.prefill(list(range(64)))   # a full context is accepted
    dm.close()
