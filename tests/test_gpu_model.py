"""Whole-model parity on the GPU: the device forward (CUDA graphs of the fused
kernels) against the oracle's restatement of the Java forward passes, on the
same seeded synthetic weights (the device generator's bytes equal the
oracle's).  Checks: logits within 1e-4 relative L2 at every step (fp32
accumulation in different orders through all layers), and the greedy token
ids identical for the first 64 generated tokens.
"""
import numpy as np
import pytest

import oracle
from brewference_b200 import config as C
from brewference_b200.api import DeviceModel

pytestmark = pytest.mark.gpu
LOGIT_TOL = 1e-4


def rel(a, b):
    return float(np.linalg.norm(a.astype(np.float64) - b) / np.linalg.norm(b.astype(np.float64)))


def small(arch, **kw):
    base = {C.ARCH_LLAMA: C.smollm2_135m, C.ARCH_QWEN3: C.qwen3_1_7b, C.ARCH_GEMMA3: C.gemma3_1b,
            C.ARCH_QWEN2: C.qwen25_7b, C.ARCH_GEMMA2: C.gemma2_2b, C.ARCH_SMOLLM3: C.smollm3_3b}[arch]()
    # SmolLM3: layer 3 is a no-RoPE layer; Gemma2: local / global layers alternate
    kw.setdefault("n_layers", 5 if arch == C.ARCH_SMOLLM3 else 3)
    kw.setdefault("vocab_size", 4096)
    kw.setdefault("seq_len", 256)
    if arch == C.ARCH_QWEN2:   # the device forward streams Q8_0/Q4_0 matrices
        kw.update(type_embed=C.TYPE_Q8_0, type_output=C.TYPE_Q8_0, type_q=C.TYPE_Q8_0, type_k=C.TYPE_Q8_0,
                  type_v=C.TYPE_Q8_0, type_o=C.TYPE_Q8_0, type_gate=C.TYPE_Q8_0, type_up=C.TYPE_Q8_0,
                  type_down=C.TYPE_Q8_0, dim=1024, hidden_dim=2048, n_heads=8, n_kv_heads=4)
    if arch in (C.ARCH_GEMMA3, C.ARCH_GEMMA2):
        kw.setdefault("sliding_window", 16)
    if arch in (C.ARCH_GEMMA2, C.ARCH_SMOLLM3):   # smaller widths, same head layout
        kw.setdefault("dim", 1024)
        kw.setdefault("hidden_dim", 2048)
    return base.replace(**kw)


def run_parity(cfg, seed, prompt_len, n_gen, check_steps=4):
    dm = DeviceModel.synthesize(cfg, seed)
    om = oracle.OracleModel(cfg, seed)
    rng = np.random.default_rng(seed)
    prompt = rng.integers(0, cfg.vocab_size, prompt_len).tolist()
    # step-by-step logits through brew_model_forward
    dm.reset()
    om.reset()
    for i in range(min(check_steps, prompt_len)):
        lg, am = dm.forward([prompt[i]], [i])
        ref = om.forward(prompt[i], i)
        assert rel(lg[0], ref) < LOGIT_TOL, (i, rel(lg[0], ref))
        assert am[0] == int(np.argmax(lg[0]))
    # greedy generation with the reference's token order
    got = dm.generate(prompt, n_gen)
    want = om.generate(prompt, n_gen)
    assert got == want
    dm.close()
    om.close()
    return got


@pytest.mark.parametrize("arch", [C.ARCH_LLAMA, C.ARCH_QWEN2, C.ARCH_QWEN3, C.ARCH_GEMMA3, C.ARCH_GEMMA2,
                                  C.ARCH_SMOLLM3])
def test_small_models_tokens_and_logits(device, arch):
    cfg = small(arch)
    run_parity(cfg, 1000 + arch, prompt_len=20, n_gen=64)


def test_untied_output_varied_tokens(device):
    """An untied classifier gives varied greedy tokens (a tied random model
    tends to repeat its input)."""
    cfg = small(C.ARCH_QWEN3, tied_embeddings=0, type_output=C.TYPE_Q8_0)
    toks = run_parity(cfg, 4242, prompt_len=12, n_gen=64)
    assert len(set(toks)) > 4


@pytest.mark.parametrize("arch", [C.ARCH_GEMMA3, C.ARCH_GEMMA2])
def test_gemma_window_crossing(device, arch):
    """Sliding-window layers (window 16) with a 40-token prompt: Gemma3's
    global layer is the 6th, Gemma2's every 2nd."""
    cfg = small(arch, n_layers=7)
    run_parity(cfg, 77, prompt_len=40, n_gen=24)


def test_batched_forward_matches_single(device):
    """Four sequences forwarded together, each with its own KV cache: every
    step's logits of every sequence against the oracle run on that sequence
    alone, and the device argmax against the logits."""
    cfg = small(C.ARCH_QWEN3)
    dm = DeviceModel.synthesize(cfg, 5, max_batch=4)
    om = oracle.OracleModel(cfg, 5)
    toks = [[3, 9, 27, 81], [4, 8, 15, 16], [1, 1, 2, 3]]
    got = []
    for step in range(len(toks)):
        lg, am = dm.forward(toks[step], [step] * 4)
        got.append(lg.copy())
        for b in range(4):
            assert am[b] == int(np.argmax(lg[b])), (step, b)
    for b in range(4):
        om.reset()
        for step in range(len(toks)):
            ref = om.forward(toks[step][b], step)
            assert rel(got[step][b], ref) < LOGIT_TOL, (step, b, rel(got[step][b], ref))
    dm.close()
    om.close()


def test_smollm2_135m_full_shape(device):
    """The SmolLM2-135M-shaped config: 32-token prompt, 64 greedy tokens."""
    cfg = C.smollm2_135m()
    run_parity(cfg, 2024, prompt_len=32, n_gen=64, check_steps=2)


def test_generate_errors_and_limits(device):
    cfg = small(C.ARCH_LLAMA, seq_len=48)
    dm = DeviceModel.synthesize(cfg, 3)
    with pytest.raises(Exception):
        dm.generate([1] * 49, 4)                  # context limit
    assert len(dm.generate([1] * 40, 0)) == 8     # max_new <= 0: remaining context
    full = dm.generate([5, 6], 6)
    dm.close()
    eos = full[3]
    dm2 = DeviceModel.synthesize(cfg.replace(eos_token=eos), 3)
    assert dm2.generate([5, 6], 6) == full[: full.index(eos) + 1]
    dm2.close()


@pytest.mark.parametrize("arch,dims,plen", [
    # head 128, 8 kv heads: 18 chunks per kv head, 56 positions each at
    # position 1000 (two rounds of staged K / V rows)
    (C.ARCH_QWEN3, {}, 1000),
    # head 64, 4 kv heads: 37 chunks, 49 positions each at position 1800
    (C.ARCH_LLAMA, dict(dim=1024, hidden_dim=2048, n_heads=16, n_kv_heads=4, head_size=64), 1800),
])
def test_long_context_attention_rounds(device, arch, dims, plen):
    """A prompt long enough that every attention chunk of the decode kernel
    takes more than one round of staged positions: the next position's
    logits and 16 greedy tokens against the oracle (prefill batched on the
    device, token by token on the oracle)."""
    from brewference_b200.api import PREFILL_BATCHED
    cfg = small(arch, seq_len=2048, **dims)
    seed = 99
    prompt = np.random.default_rng(seed).integers(0, cfg.vocab_size, plen).astype(np.int32)
    om = oracle.OracleModel(cfg, seed)
    om.reset()
    for i, t in enumerate(prompt):
        om.forward(int(t), i)
    pending, pos, want, ref = int(prompt[-1]), plen, [], None
    for _ in range(16):
        lg = om.forward(pending, pos)
        if ref is None:
            ref = lg.copy()
        pending, pos = oracle.argmax(lg), pos + 1
        want.append(pending)
    om.close()
    dm = DeviceModel.synthesize(cfg, seed)
    dm.set_prefill(PREFILL_BATCHED)
    dm.prefill(prompt)
    lg, _ = dm.forward([int(prompt[-1])], [plen])
    assert rel(lg[0], ref) < LOGIT_TOL, rel(lg[0], ref)
    assert dm.generate(prompt, 16) == want
    dm.close()


@pytest.mark.parametrize("arch", [C.ARCH_QWEN3, C.ARCH_GEMMA2])
def test_forward_argmax_only_call(device, arch):
    """brew_model_forward without a logits buffer, one sequence: the token
    and position go to the decode kernel as launch parameters and the id
    comes back through mapped host memory.  Calls without and with logits
    alternate on one model; every step's id must equal the oracle's argmax
    (and the device argmax of the logits on the logits steps)."""
    cfg = small(arch)
    seed = 31 + arch
    dm = DeviceModel.synthesize(cfg, seed)
    om = oracle.OracleModel(cfg, seed)
    dm.reset()
    om.reset()
    toks = np.random.default_rng(seed).integers(0, cfg.vocab_size, 24).tolist()
    for i, t in enumerate(toks):
        ref = om.forward(t, i)
        if i % 3 == 2:
            lg, am = dm.forward([t], [i])
            assert rel(lg[0], ref) < LOGIT_TOL, (i, rel(lg[0], ref))
            assert am[0] == int(np.argmax(lg[0])), i
        else:
            lg, am = dm.forward([t], [i], want_logits=False)
            assert lg is None
        assert am[0] == oracle.argmax(ref), i
    with pytest.raises(Exception):   # rejected on the host, before any launch
        dm.forward([cfg.vocab_size], [len(toks)], want_logits=False)
    _, am = dm.forward([toks[0]], [len(toks)], want_logits=False)
    assert 0 <= am[0] < cfg.vocab_size
    dm.close()
    om.close()
