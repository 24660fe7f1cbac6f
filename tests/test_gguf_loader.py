"""GGUF reading without a GPU: brew_gguf_open / brew_gguf_config /
brew_gguf_tensor_info against a seeded file written by gguf-py's GGUFWriter
and read back by gguf-py's GGUFReader (gguf 0.19.0).

What the reference does (gguf/Reader.java:25-125,
gguf/GgufConfigParser.java:9-59, the per-architecture CheckpointLoaders and
gguf/GgufWeightsLoader.java:159-162) is what the library must reproduce:
the config fields, the head-size rules, the vocabulary size from the token
list, the tied classifier when output.weight is absent, the tensor infos and
the aligned data offset; and the same IOExceptions for a bad magic number, an
unsupported version or a truncated file.
"""
import os

import numpy as np
import pytest
from gguf import GGUFReader

import oracle
from brewference_b200 import _native as N
from brewference_b200 import config as C
from brewference_b200.api import GgufFile
from tests import gguf_fixture


def small(arch, **kw):
    base = {C.ARCH_LLAMA: C.smollm2_135m, C.ARCH_QWEN2: C.qwen25_7b, C.ARCH_QWEN3: C.qwen3_1_7b,
            C.ARCH_GEMMA3: C.gemma3_1b, C.ARCH_GEMMA2: C.gemma2_2b, C.ARCH_SMOLLM3: C.smollm3_3b}[arch]()
    kw.setdefault("n_layers", 2)
    kw.setdefault("vocab_size", 512)
    kw.setdefault("seq_len", 128)
    kw.setdefault("eos_token", 511)
    kw.setdefault("dim", 256)
    kw.setdefault("hidden_dim", 512)
    return base.replace(**kw)


CASES = {
    "llama-untied": small(C.ARCH_LLAMA, n_heads=4, n_kv_heads=2, head_size=64, tied_embeddings=0),
    "qwen2-bias-q4": small(C.ARCH_QWEN2, n_heads=2, n_kv_heads=1, head_size=128, tied_embeddings=1,
                           type_embed=C.TYPE_Q8_0, type_output=C.TYPE_Q8_0, type_q=C.TYPE_Q4_0, type_k=C.TYPE_Q4_0,
                           type_v=C.TYPE_Q4_0, type_o=C.TYPE_Q8_0, type_gate=C.TYPE_Q4_0, type_up=C.TYPE_Q4_0,
                           type_down=C.TYPE_Q8_0),
    "qwen3-qknorm": small(C.ARCH_QWEN3, n_heads=4, n_kv_heads=2),
    "gemma3-window": small(C.ARCH_GEMMA3, n_heads=2, n_kv_heads=1, sliding_window=8, n_layers=3),
    "gemma2": small(C.ARCH_GEMMA2, n_heads=2, n_kv_heads=1, sliding_window=8),
    "smollm3": small(C.ARCH_SMOLLM3, n_heads=2, n_kv_heads=1, n_layers=4),
    "kquant": small(C.ARCH_QWEN2, n_heads=2, n_kv_heads=1, tied_embeddings=0, type_embed=C.TYPE_Q4_K,
                    type_output=C.TYPE_Q6_K, type_q=C.TYPE_Q4_K, type_k=C.TYPE_Q4_K, type_v=C.TYPE_Q4_K,
                    type_o=C.TYPE_Q4_K, type_gate=C.TYPE_Q4_K, type_up=C.TYPE_Q4_K, type_down=C.TYPE_Q6_K),
}


def write_case(tmp_path, key, seed=11):
    cfg = CASES[key]
    om = oracle.OracleModel(cfg, seed)
    gguf_fixture.randomize_vectors(om, seed)
    path = str(tmp_path / f"{key}.gguf")
    gguf_fixture.write(path, cfg, om)
    return cfg, om, path


@pytest.mark.parametrize("key", sorted(CASES))
def test_config_and_tensor_infos_match_gguf_py(tmp_path, key):
    cfg, om, path = write_case(tmp_path, key)
    om.close()
    with GgufFile(path) as g:
        got = g.config()
        infos = g.tensors()
    for f in ("arch", "dim", "hidden_dim", "n_layers", "n_heads", "n_kv_heads", "head_size", "vocab_size",
              "seq_len", "sliding_window", "bos_token", "eos_token", "tied_embeddings", "type_embed", "type_q",
              "type_k", "type_v", "type_o", "type_gate", "type_up", "type_down"):
        assert getattr(got, f) == getattr(cfg, f), f
    assert got.type_output == (cfg.type_embed if cfg.tied_embeddings else cfg.type_output)
    assert got.eps == pytest.approx(cfg.eps, rel=1e-7)
    assert got.rope_base == pytest.approx(cfg.rope_base)
    r = GGUFReader(path)
    ref = {t.name: (int(t.tensor_type), int(t.n_elements), int(t.data_offset)) for t in r.tensors}
    assert len(infos) == len(ref)
    for name, t, n, off in infos:
        assert ref[name] == (t, n, off), name


def test_vectors_f16_and_f32_are_as_written(tmp_path):
    """readFloatArray (GgufWeightsLoader.java:249-278): the raw bytes at the
    reported offsets decode to the oracle's vectors, F32 and F16 layers."""
    cfg, om, path = write_case(tmp_path, "qwen3-qknorm")
    raw = np.fromfile(path, np.uint8)
    with GgufFile(path) as g:
        infos = {name: (t, n, off) for name, t, n, off in g.tensors()}
    att = om.vector(0)
    for l in range(cfg.n_layers):
        t, n, off = infos[f"blk.{l}.attn_norm.weight"]
        if t == C.TYPE_F32:
            v = raw[off:off + 4 * n].view(np.float32)
        else:
            assert t == C.TYPE_F16 and l % 2 == 1
            v = raw[off:off + 2 * n].view(np.float16).astype(np.float32)
        np.testing.assert_array_equal(v, att[l * cfg.dim:(l + 1) * cfg.dim])
    om.close()


def test_io_errors(tmp_path):
    cfg, om, path = write_case(tmp_path, "llama-untied")
    om.close()
    data = bytearray(open(path, "rb").read())
    bad = tmp_path / "bad_magic.gguf"
    bad.write_bytes(b"GGUX" + bytes(data[4:]))
    with pytest.raises(N.BrewError) as e:
        GgufFile(str(bad))
    assert e.value.code == N.ERR_IO and "magic" in str(e.value)
    ver = tmp_path / "bad_version.gguf"
    ver.write_bytes(bytes(data[:4]) + (7).to_bytes(4, "little") + bytes(data[8:]))
    with pytest.raises(N.BrewError) as e:
        GgufFile(str(ver))
    assert e.value.code == N.ERR_IO and "version" in str(e.value)
    cut = tmp_path / "truncated.gguf"
    cut.write_bytes(bytes(data[: len(data) // 2]))
    with pytest.raises(N.BrewError) as e:
        GgufFile(str(cut))
    assert e.value.code == N.ERR_IO
    with pytest.raises(N.BrewError) as e:
        GgufFile(str(tmp_path / "missing.gguf"))
    assert e.value.code == N.ERR_IO


def test_unsupported_architecture(tmp_path):
    """ModelRunnerFactory.createModelRunner (model/ModelRunnerFactory.java:46-47)
    rejects other architectures; so does the config."""
    from gguf import GGUFWriter
    p = str(tmp_path / "phi3.gguf")
    w = GGUFWriter(p, "phi3")
    w.add_uint32("phi3.embedding_length", 64)
    w.add_array("tokenizer.ggml.tokens", ["a", "b"])
    w.add_tensor("token_embd.weight", np.zeros((2, 64), np.float32))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    with GgufFile(p) as g:
        with pytest.raises(N.BrewError) as e:
            g.config()
    assert e.value.code == N.ERR_UNSUPPORTED and "phi3" in str(e.value)
