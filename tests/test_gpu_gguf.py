"""Models loaded from GGUF files on the GPU, against the oracle fed the same
bytes.

A seeded GGUF v3 (gguf-py's GGUFWriter, tests/gguf_fixture.py) holds the
oracle's packed blocks and seeded non-trivial norm / bias vectors (F32, and
F16 on odd layers).  Two routes into the device are checked:
  * brew_model_load_gguf: the one-call loader (GgufCheckpointLoader.loadWeights
    + GgufWeightsLoader.load, gguf/GgufWeightsLoader.java:24-165);
  * the boundary a Java host drives itself: the file's tensors parsed the way
    gguf/Reader.java:25-81 does (brew_gguf_tensor_info), each packed tensor
    uploaded with brew_tensor_upload, the vectors decoded as readFloatArray
    does (:249-278), and the model built with brew_model_create.
Bar: logits within 1e-4 relative L2 of the oracle's at every checked step and
the first 64 greedy tokens identical (runtime/ModelRunner.java:122-206).
"""
import numpy as np
import pytest

import oracle
from brewference_b200 import config as C
from brewference_b200.api import DeviceModel, GgufFile, PackedTensor
from tests import gguf_fixture
from tests.test_gguf_loader import CASES, write_case

pytestmark = pytest.mark.gpu
LOGIT_TOL = 1e-4


def rel(a, b):
    return float(np.linalg.norm(a.astype(np.float64) - b) / np.linalg.norm(b.astype(np.float64)))


def check(dm, om, cfg, seed, n_gen=64, steps=3):
    prompt = np.random.default_rng(seed).integers(0, cfg.vocab_size, 12).tolist()
    dm.reset()
    om.reset()
    for i in range(steps):
        lg, am = dm.forward([prompt[i]], [i])
        ref = om.forward(prompt[i], i)
        assert rel(lg[0], ref) < LOGIT_TOL, (i, rel(lg[0], ref))
        assert am[0] == int(np.argmax(lg[0]))
    got = dm.generate(prompt, n_gen)
    want = om.generate(prompt, n_gen)
    assert got == want


@pytest.mark.parametrize("key", sorted(CASES))
def test_load_gguf_matches_oracle(device, tmp_path, key):
    cfg, om, path = write_case(tmp_path, key, seed=21)
    dm = DeviceModel.load_gguf(path)
    assert dm.cfg.arch == cfg.arch and dm.cfg.vocab_size == cfg.vocab_size
    check(dm, om, cfg, 21)
    dm.close()
    om.close()


def parse_and_create(path):
    """The host-driven route: Reader-style tensor list, brew_tensor_upload of
    the packed bytes (layers concatenated, GgufWeightsLoader.java:139-145),
    readFloatArray of the vectors, brew_model_create."""
    raw = np.fromfile(path, np.uint8)
    with GgufFile(path) as g:
        cfg = g.config()
        infos = {name: (t, n, off) for name, t, n, off in g.tensors()}

    def packed(name):
        t, n, off = infos[name]
        eb, bb = C.TYPE_BLOCK[t]
        return t, n, raw[off:off + n // eb * bb]

    def floats(name):
        t, n, off = infos[name]
        if t == C.TYPE_F32:
            return raw[off:off + 4 * n].view(np.float32).copy()
        assert t == C.TYPE_F16, name
        return raw[off:off + 2 * n].view(np.float16).astype(np.float32)

    tensors = {}
    t, n, b = packed("token_embd.weight")
    tensors["token_embd"] = PackedTensor.upload(t, b, n)
    if "output.weight" in infos:
        t, n, b = packed("output.weight")
        tensors["output"] = PackedTensor.upload(t, b, n)
    fams = {"wq": "attn_q.weight", "wk": "attn_k.weight", "wv": "attn_v.weight", "wo": "attn_output.weight",
            "w_gate": "ffn_gate.weight", "w_up": "ffn_up.weight", "w_down": "ffn_down.weight"}
    for key, tail in fams.items():
        parts = [packed(f"blk.{l}.{tail}") for l in range(cfg.n_layers)]
        tensors[key] = PackedTensor.upload(parts[0][0], np.concatenate([p[2] for p in parts]),
                                           sum(p[1] for p in parts))
    vecs = {"rms_att": "attn_norm.weight", "rms_ffn": "ffn_norm.weight", "post_att": "post_attention_norm.weight",
            "post_ffn": "post_ffw_norm.weight", "rms_q": "attn_q_norm.weight", "rms_k": "attn_k_norm.weight",
            "q_bias": "attn_q.bias", "k_bias": "attn_k.bias", "v_bias": "attn_v.bias"}
    vectors = {"rms_final": floats("output_norm.weight")}
    for key, tail in vecs.items():
        if f"blk.0.{tail}" in infos:
            vectors[key] = np.concatenate([floats(f"blk.{l}.{tail}") for l in range(cfg.n_layers)])
    return DeviceModel.create(cfg, tensors, vectors), tensors


@pytest.mark.parametrize("key", ["qwen3-qknorm", "qwen2-bias-q4", "gemma3-window", "kquant"])
def test_host_parsed_upload_and_model_create(device, tmp_path, key):
    cfg, om, path = write_case(tmp_path, key, seed=33)
    dm, tensors = parse_and_create(path)
    check(dm, om, cfg, 33)
    dm.close()
    for t in tensors.values():
        t.free()
    om.close()
