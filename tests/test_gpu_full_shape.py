"""Parity at the full shapes of the benchmarked configurations (not the
reduced stand-ins of the other model tests):

  * Qwen3-1.7B-shaped, Q8_0, 28 layers, vocabulary 151936, context 4096:
    a 512-token seeded prompt through both prefill modes (token by token, the
    reference's ModelRunner.prefill order, and the batched tcgen05 prefill);
    the next position's logits within 1e-4 relative L2 of the oracle's and
    the first 64 greedy tokens identical to the oracle's
    (runtime/ModelRunner.java:122-206).
  * Gemma-3-1B-shaped: Q4_0 layers, Q8_0 tied embedding, vocabulary 262144,
    sliding window 512 (5 of 6 layers): a 600-token prompt, so the window
    binds, checked the same way.
  * Qwen2.5-7B-shaped, all 28 layers, Q4_K / Q6_K, 32 concurrent sequences:
    sequence 0 against the oracle, and sequences forwarded together against
    the same sequences forwarded alone.

The oracle runs on all host threads; the whole file stays within a few
minutes of oracle time.
"""
import numpy as np
import pytest

import oracle
from brewference_b200 import config as C
from brewference_b200.api import PREFILL_BATCHED, PREFILL_TOKENS, DeviceModel

pytestmark = pytest.mark.gpu
LOGIT_TOL = 1e-4


def rel(a, b):
    return float(np.linalg.norm(a.astype(np.float64) - b) / np.linalg.norm(b.astype(np.float64)))


def oracle_session(cfg, seed, prompt, n_gen):
    """ModelRunner.prefill + greedy sampleNextToken on the oracle: the logits
    of the first generated position and the generated ids."""
    om = oracle.OracleModel(cfg, seed)
    om.reset()
    for i, t in enumerate(prompt):
        om.forward(int(t), i)
    pending, pos, toks, first = int(prompt[-1]), len(prompt), [], None
    for _ in range(n_gen):
        lg = om.forward(pending, pos)
        if first is None:
            first = lg.copy()
        tok = oracle.argmax(lg)
        toks.append(tok)
        pending, pos = tok, pos + 1
    om.close()
    return first, toks


def device_session(dm, prompt, n_gen, mode):
    dm.set_prefill(mode)
    dm.prefill(prompt)
    lg, _ = dm.forward([int(prompt[-1])], [len(prompt)])
    toks = dm.generate(prompt, n_gen)
    return lg[0], toks


@pytest.mark.parametrize("name", ["qwen3-1.7b", "gemma3-1b"])
def test_full_shape_prompt_and_64_greedy_tokens(device, name):
    cfg = {"qwen3-1.7b": C.qwen3_1_7b, "gemma3-1b": C.gemma3_1b}[name]()
    plen = 512 if name == "qwen3-1.7b" else 600
    seed = 4242
    prompt = np.random.default_rng(seed).integers(0, cfg.vocab_size, plen).astype(np.int32)
    ref_logits, ref_toks = oracle_session(cfg, seed, prompt, 64)
    dm = DeviceModel.synthesize(cfg, seed)
    for mode in (PREFILL_TOKENS, PREFILL_BATCHED):
        lg, toks = device_session(dm, prompt, 64, mode)
        assert rel(lg, ref_logits) < LOGIT_TOL, (name, mode, rel(lg, ref_logits))
        assert toks == ref_toks, (name, mode, toks[:8], ref_toks[:8])
    dm.close()


def test_qwen25_7b_full_depth_32_sequences(device):
    cfg = C.qwen25_7b()
    B, steps, seed = 32, 4, 606
    toks = np.random.default_rng(seed).integers(0, cfg.vocab_size, (steps, B)).astype(np.int32)
    dm = DeviceModel.synthesize(cfg, seed, max_batch=B)
    batched = []
    for pos in range(steps):
        lg, am = dm.forward(toks[pos], np.full(B, pos, np.int32))
        assert all(am[b] == int(np.argmax(lg[b])) for b in range(B))
        batched.append(lg.copy())
    # each sequence's cache is its own: a sequence alone gives the same logits
    for b in (1, 17, 31):
        dm.reset()
        for pos in range(steps):
            lg, _ = dm.forward([toks[pos][b]], [pos])
            assert rel(batched[pos][b], lg[0]) < 1e-6, (b, pos)
    dm.close()
    om = oracle.OracleModel(cfg, seed)
    om.reset()
    for pos in range(steps):
        ref = om.forward(int(toks[pos][0]), pos)
        assert rel(batched[pos][0], ref) < LOGIT_TOL, (pos, rel(batched[pos][0], ref))
    om.close()
