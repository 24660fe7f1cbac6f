"""Writes seeded synthetic GGUF v3 checkpoints with gguf-py's GGUFWriter
(gguf 0.19.0, GGML's own Python writer) for the loader tests.

The weights are the oracle's synthetic model (the same seeded packed blocks),
with its norm and bias vectors replaced by seeded random values, so that the
oracle and a model loaded from the file compute the same forward pass.  The
metadata keys are those gguf/GgufConfigParser.java:9-59 reads, the tensor
names those gguf/GgufWeightsLoader.java:62-136 matches.  Norm vectors of odd
layers are written as F16 (readFloatArray's second branch, :264-271); the
oracle then holds their fp16-rounded values.

Test infrastructure: only tests/ imports it.
"""
from __future__ import annotations

import numpy as np
from gguf import GGMLQuantizationType as QT
from gguf import GGUFWriter

import oracle
from brewference_b200 import config as C

QTYPE = {C.TYPE_Q8_0: QT.Q8_0, C.TYPE_Q4_0: QT.Q4_0, C.TYPE_Q4_K: QT.Q4_K, C.TYPE_Q6_K: QT.Q6_K}
ARCH = {C.ARCH_LLAMA: "llama", C.ARCH_QWEN2: "qwen2", C.ARCH_QWEN3: "qwen3", C.ARCH_GEMMA3: "gemma3",
        C.ARCH_GEMMA2: "gemma2", C.ARCH_SMOLLM3: "smollm3"}
# oracle vector index -> (GGUF tensor name tail, per-layer?)
VECTORS = {0: ("attn_norm.weight", True), 1: ("ffn_norm.weight", True), 2: ("output_norm.weight", False),
           3: ("post_attention_norm.weight", True), 4: ("post_ffw_norm.weight", True),
           5: ("attn_q_norm.weight", True), 6: ("attn_k_norm.weight", True), 7: ("attn_q.bias", True),
           8: ("attn_k.bias", True), 9: ("attn_v.bias", True)}
MATRICES = {C.W_Q: "attn_q.weight", C.W_K: "attn_k.weight", C.W_V: "attn_v.weight", C.W_O: "attn_output.weight",
            C.W_GATE: "ffn_gate.weight", C.W_UP: "ffn_up.weight", C.W_DOWN: "ffn_down.weight"}


def randomize_vectors(om: "oracle.OracleModel", seed: int) -> None:
    """Seeded non-trivial norm weights (1 + N(0, 0.1)) and biases (N(0, 0.02))
    in the oracle model; odd layers' norm weights rounded to fp16."""
    cfg = om.cfg
    rng = np.random.default_rng(seed)
    for vi, (tail, layered) in VECTORS.items():
        v = om.vector(vi)
        if v is None:
            continue
        if vi >= 7:
            v[:] = rng.normal(0.0, 0.02, v.size).astype(np.float32)
            continue
        v[:] = (1.0 + rng.normal(0.0, 0.1, v.size)).astype(np.float32)
        if layered:
            per = v.size // cfg.n_layers
            for l in range(1, cfg.n_layers, 2):
                seg = v[l * per:(l + 1) * per]
                seg[:] = seg.astype(np.float16).astype(np.float32)


def write(path: str, cfg: C.ModelConfig, om: "oracle.OracleModel", context_length: int | None = None) -> None:
    arch = ARCH[cfg.arch]
    w = GGUFWriter(path, arch)
    w.add_name("synthetic " + cfg.name)
    w.add_uint32(f"{arch}.embedding_length", cfg.dim)
    w.add_uint32(f"{arch}.feed_forward_length", cfg.hidden_dim)
    w.add_uint32(f"{arch}.block_count", cfg.n_layers)
    w.add_uint32(f"{arch}.context_length", context_length or cfg.seq_len)
    w.add_uint32(f"{arch}.attention.head_count", cfg.n_heads)
    w.add_uint32(f"{arch}.attention.head_count_kv", cfg.n_kv_heads)
    w.add_float32(f"{arch}.attention.layer_norm_rms_epsilon", cfg.eps)
    if cfg.sliding_window:
        w.add_uint32(f"{arch}.attention.sliding_window", cfg.sliding_window)
    if cfg.rope_base > 0:
        w.add_float32(f"{arch}.rope.freq_base", cfg.rope_base)
    w.add_string("tokenizer.ggml.model", "gpt2")
    w.add_array("tokenizer.ggml.tokens", [f"<t{i}>" for i in range(cfg.vocab_size)])
    w.add_uint32("tokenizer.ggml.bos_token_id", cfg.bos_token)
    w.add_uint32("tokenizer.ggml.eos_token_id", cfg.eos_token if cfg.eos_token >= 0 else cfg.vocab_size - 1)

    def matrix(name, which, layer, layers):
        rows, cols, t, _ = cfg.matrix_shapes()[which]
        data = om.tensor(which)
        per = data.size // layers
        blob = np.ascontiguousarray(data[layer * per:(layer + 1) * per]).reshape(rows, per // rows)
        w.add_tensor(name, blob, raw_dtype=QTYPE[t])

    matrix("token_embd.weight", C.W_EMBED, 0, 1)
    if not cfg.tied_embeddings:
        matrix("output.weight", C.W_OUTPUT, 0, 1)
    for vi, (tail, layered) in VECTORS.items():
        v = om.vector(vi)
        if v is None:
            continue
        if not layered:
            w.add_tensor(tail, np.array(v, np.float32))
            continue
        per = v.size // cfg.n_layers
        for l in range(cfg.n_layers):
            seg = np.array(v[l * per:(l + 1) * per], np.float32)
            f16 = vi < 7 and l % 2 == 1
            w.add_tensor(f"blk.{l}.{tail}", seg.astype(np.float16) if f16 else seg)
    for l in range(cfg.n_layers):
        for which, tail in MATRICES.items():
            matrix(f"blk.{l}.{tail}", which, l, cfg.n_layers)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
