"""Model hyper-parameters (the fields of the reference's gguf/Config.java that
the forward pass reads) as the ctypes mirror of ``brew_config`` in
include/brew.h, plus shape presets for the architectures this path serves.

The presets describe *shapes* only; weights come from a GGUF file or from the
seeded synthetic generator.  Synthetic presets use ``eos_token = -1`` so a
greedy decode runs for its full length (a random-weight model would otherwise
stop whenever it happens to emit the checkpoint's EOS id).
"""
from __future__ import annotations

import ctypes
import dataclasses

TYPE_F32, TYPE_F16, TYPE_Q4_0, TYPE_Q8_0, TYPE_Q4_K, TYPE_Q6_K = 0, 1, 2, 8, 12, 14
TYPE_NAMES = {0: "F32", 1: "F16", 2: "Q4_0", 8: "Q8_0", 12: "Q4_K", 14: "Q6_K"}
# (elements per block, bytes per block) of each GGML type
TYPE_BLOCK = {0: (1, 4), 1: (1, 2), 2: (32, 18), 8: (32, 34), 12: (256, 144), 14: (256, 210)}

ARCH_LLAMA, ARCH_QWEN2, ARCH_QWEN3, ARCH_GEMMA3, ARCH_GEMMA2, ARCH_SMOLLM3 = 0, 1, 2, 3, 4, 5
# general.architecture values the reference's ModelRunnerFactory accepts
# (model/ModelRunnerFactory.java:29-47); "llama2" runs the llama graph
ARCH_NAMES = {0: "llama", 1: "qwen2", 2: "qwen3", 3: "gemma3", 4: "gemma2", 5: "smollm3"}
ARCH_IDS = {"llama": 0, "llama2": 0, "qwen2": 1, "qwen3": 2, "gemma3": 3, "gemma2": 4, "smollm3": 5}

# tensor indices used by brew_model_tensor / the synthetic generator
W_EMBED, W_OUTPUT, W_Q, W_K, W_V, W_O, W_GATE, W_UP, W_DOWN = range(9)


class BrewConfig(ctypes.Structure):
    _fields_ = [
        ("arch", ctypes.c_int32), ("dim", ctypes.c_int32), ("hidden_dim", ctypes.c_int32),
        ("n_layers", ctypes.c_int32), ("n_heads", ctypes.c_int32), ("n_kv_heads", ctypes.c_int32),
        ("head_size", ctypes.c_int32), ("vocab_size", ctypes.c_int32), ("seq_len", ctypes.c_int32),
        ("sliding_window", ctypes.c_int32), ("eps", ctypes.c_float), ("rope_base", ctypes.c_float),
        ("rope_scale", ctypes.c_float), ("bos_token", ctypes.c_int32), ("eos_token", ctypes.c_int32),
        ("tied_embeddings", ctypes.c_int32),
        ("type_embed", ctypes.c_int32), ("type_output", ctypes.c_int32),
        ("type_q", ctypes.c_int32), ("type_k", ctypes.c_int32), ("type_v", ctypes.c_int32),
        ("type_o", ctypes.c_int32), ("type_gate", ctypes.c_int32), ("type_up", ctypes.c_int32),
        ("type_down", ctypes.c_int32),
    ]


@dataclasses.dataclass
class ModelConfig:
    arch: int
    dim: int
    hidden_dim: int
    n_layers: int
    n_heads: int
    n_kv_heads: int
    head_size: int
    vocab_size: int
    seq_len: int
    eps: float
    rope_base: float = 0.0
    rope_scale: float = 0.0
    sliding_window: int = 0
    bos_token: int = 1
    eos_token: int = -1
    tied_embeddings: int = 1
    type_embed: int = TYPE_Q8_0
    type_output: int = TYPE_Q8_0
    type_q: int = TYPE_Q8_0
    type_k: int = TYPE_Q8_0
    type_v: int = TYPE_Q8_0
    type_o: int = TYPE_Q8_0
    type_gate: int = TYPE_Q8_0
    type_up: int = TYPE_Q8_0
    type_down: int = TYPE_Q8_0
    name: str = ""

    def to_c(self) -> BrewConfig:
        c = BrewConfig()
        for f, _ in BrewConfig._fields_:
            setattr(c, f, getattr(self, f))
        return c

    def replace(self, **kw) -> "ModelConfig":
        return dataclasses.replace(self, **kw)

    # ---- derived sizes --------------------------------------------------
    @property
    def q_width(self) -> int:
        return self.n_heads * self.head_size

    @property
    def kv_dim(self) -> int:
        return self.n_kv_heads * self.head_size

    def matrix_shapes(self) -> dict:
        """(rows, cols, type, layers) of each weight family."""
        out_type = self.type_embed if self.tied_embeddings else self.type_output
        return {
            W_EMBED: (self.vocab_size, self.dim, self.type_embed, 1),
            W_OUTPUT: (self.vocab_size, self.dim, out_type, 1),
            W_Q: (self.q_width, self.dim, self.type_q, self.n_layers),
            W_K: (self.kv_dim, self.dim, self.type_k, self.n_layers),
            W_V: (self.kv_dim, self.dim, self.type_v, self.n_layers),
            W_O: (self.dim, self.q_width, self.type_o, self.n_layers),
            W_GATE: (self.hidden_dim, self.dim, self.type_gate, self.n_layers),
            W_UP: (self.hidden_dim, self.dim, self.type_up, self.n_layers),
            W_DOWN: (self.dim, self.hidden_dim, self.type_down, self.n_layers),
        }

    def decode_weight_bytes(self) -> int:
        """Packed weight bytes one decode step streams: every layer matrix
        plus the classifier (the embedding row read is excluded)."""
        total = 0
        for w, (rows, cols, t, layers) in self.matrix_shapes().items():
            if w == W_EMBED:
                continue
            be, bb = TYPE_BLOCK[t]
            total += rows * cols // be * bb * layers
        return total


def smollm2_135m(**kw) -> ModelConfig:
    """Llama-arch model shaped like SmolLM2-135M, all Q8_0."""
    return ModelConfig(arch=ARCH_LLAMA, dim=576, hidden_dim=1536, n_layers=30, n_heads=9, n_kv_heads=3,
                       head_size=64, vocab_size=49152, seq_len=2048, eps=1e-5, rope_base=100000.0,
                       name="smollm2-135m-shaped", **kw)


def qwen3_1_7b(**kw) -> ModelConfig:
    """Qwen3-1.7B-shaped model, Q8_0, per-head QK RMSNorm, RoPE theta 1e6."""
    return ModelConfig(arch=ARCH_QWEN3, dim=2048, hidden_dim=6144, n_layers=28, n_heads=16, n_kv_heads=8,
                       head_size=128, vocab_size=151936, seq_len=4096, eps=1e-6, rope_base=1e6,
                       name="qwen3-1.7b-shaped", **kw)


def gemma3_1b(**kw) -> ModelConfig:
    """Gemma-3-1B-shaped model: Q4_0 layers, Q8_0 (tied) embeddings, sliding
    window 512 on 5 of 6 layers, RoPE from the architecture fallbacks."""
    return ModelConfig(arch=ARCH_GEMMA3, dim=1152, hidden_dim=6912, n_layers=26, n_heads=4, n_kv_heads=1,
                       head_size=256, vocab_size=262144, seq_len=4096, eps=1e-6, rope_base=0.0,
                       sliding_window=512, type_q=TYPE_Q4_0, type_k=TYPE_Q4_0, type_v=TYPE_Q4_0,
                       type_o=TYPE_Q4_0, type_gate=TYPE_Q4_0, type_up=TYPE_Q4_0, type_down=TYPE_Q4_0,
                       name="gemma3-1b-shaped", **kw)


def qwen25_7b(**kw) -> ModelConfig:
    """Qwen2.5-7B-shaped model: Q4_K attention/FFN, Q6_K ffn_down and output,
    QKV bias, untied output."""
    return ModelConfig(arch=ARCH_QWEN2, dim=3584, hidden_dim=18944, n_layers=28, n_heads=28, n_kv_heads=4,
                       head_size=128, vocab_size=152064, seq_len=4096, eps=1e-6, rope_base=1e6,
                       tied_embeddings=0, type_embed=TYPE_Q4_K, type_output=TYPE_Q6_K,
                       type_q=TYPE_Q4_K, type_k=TYPE_Q4_K, type_v=TYPE_Q4_K, type_o=TYPE_Q4_K,
                       type_gate=TYPE_Q4_K, type_up=TYPE_Q4_K, type_down=TYPE_Q6_K,
                       name="qwen2.5-7b-shaped", **kw)


def gemma2_2b(**kw) -> ModelConfig:
    """Gemma-2-2B-shaped model, Q8_0: head size 256 (hard-coded by the
    reference's Gemma2CheckpointLoader), sliding window 4096 on every other
    layer, GeGLU, pre/post norms."""
    return ModelConfig(arch=ARCH_GEMMA2, dim=2304, hidden_dim=9216, n_layers=26, n_heads=8, n_kv_heads=4,
                       head_size=256, vocab_size=256000, seq_len=8192, eps=1e-6, rope_base=0.0,
                       sliding_window=4096, name="gemma2-2b-shaped", **kw)


def smollm3_3b(**kw) -> ModelConfig:
    """SmolLM3-3B-shaped model, Q8_0: Llama layout (q and wo are dim x dim),
    no RoPE on every 4th layer."""
    return ModelConfig(arch=ARCH_SMOLLM3, dim=2048, hidden_dim=11008, n_layers=36, n_heads=16, n_kv_heads=4,
                       head_size=128, vocab_size=128256, seq_len=4096, eps=1e-6, rope_base=0.0,
                       name="smollm3-3b-shaped", **kw)


def llama2_7b(**kw) -> ModelConfig:
    """Llama-2-7B-shaped model, Q8_0, untied output (the reference's largest
    published Q8_0 run)."""
    return ModelConfig(arch=ARCH_LLAMA, dim=4096, hidden_dim=11008, n_layers=32, n_heads=32, n_kv_heads=32,
                       head_size=128, vocab_size=32000, seq_len=4096, eps=1e-5, rope_base=0.0,
                       tied_embeddings=0, name="llama2-7b-shaped", **kw)


PRESETS = {
    "smollm2-135m": smollm2_135m,
    "qwen3-1.7b": qwen3_1_7b,
    "gemma3-1b": gemma3_1b,
    "qwen2.5-7b": qwen25_7b,
    "gemma2-2b": gemma2_2b,
    "smollm3-3b": smollm3_3b,
    "llama2-7b": llama2_7b,
}
