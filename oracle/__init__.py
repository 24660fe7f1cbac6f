"""ctypes binding of the CPU oracle (libbrew_oracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py, as the checker.  The oracle restates the
reference's Java arithmetic (see brew_oracle.c for the file:line citations);
its block formats are pinned to gguf-py 0.19.0 by tests/golden/.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

from brewference_b200.config import BrewConfig, ModelConfig, TYPE_BLOCK

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libbrew_oracle.so")
_lib = None

_f32p = ctypes.POINTER(ctypes.c_float)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_i32p = ctypes.POINTER(ctypes.c_int32)


def build(force: bool = False) -> str:
    if force or not os.path.exists(_LIB_PATH):
        subprocess.check_call(["make", "-s", "-C", _HERE])
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(_LIB_PATH)
        L.ob_half_to_float.restype = ctypes.c_float
        L.ob_half_to_float.argtypes = [ctypes.c_uint16]
        L.ob_float_to_half.restype = ctypes.c_uint16
        L.ob_float_to_half.argtypes = [ctypes.c_float]
        L.ob_set_threads.argtypes = [ctypes.c_int]
        L.ob_get_threads.restype = ctypes.c_int
        L.ob_synth_value.restype = ctypes.c_float
        L.ob_synth_value.argtypes = [ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_float]
        L.ob_synth_fill.argtypes = [ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_int64,
                                    ctypes.c_float, _f32p]
        L.ob_quantize.argtypes = [ctypes.c_int, _f32p, ctypes.c_int64, _u8p]
        L.ob_dequantize.argtypes = [ctypes.c_int, _u8p, ctypes.c_int64, ctypes.c_int64, _f32p]
        L.ob_synth_quantized.argtypes = [ctypes.c_int, ctypes.c_uint64, ctypes.c_uint32, ctypes.c_int64,
                                         ctypes.c_float, _u8p]
        L.ob_matvec.argtypes = [ctypes.c_int, _u8p, ctypes.c_int64, _f32p, _f32p, ctypes.c_int, ctypes.c_int]
        L.ob_rmsnorm.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int, ctypes.c_float]
        L.ob_headwise_rmsnorm.argtypes = [_f32p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_float]
        L.ob_softmax.argtypes = [_f32p, ctypes.c_int]
        L.ob_argmax.restype = ctypes.c_int
        L.ob_argmax.argtypes = [_f32p, ctypes.c_int]
        L.ob_rope.argtypes = [_f32p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float,
                              ctypes.c_float, ctypes.c_int]
        L.ob_glu.argtypes = [_f32p, _f32p, ctypes.c_int, ctypes.c_int]
        L.ob_model_synth.restype = ctypes.c_void_p
        L.ob_model_synth.argtypes = [ctypes.POINTER(BrewConfig), ctypes.c_uint64]
        L.ob_model_free.argtypes = [ctypes.c_void_p]
        L.ob_model_tensor.restype = ctypes.c_void_p
        L.ob_model_tensor.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ctypes.c_int64)]
        L.ob_model_vector.restype = ctypes.c_void_p
        L.ob_model_vector.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ctypes.c_int64)]
        L.ob_model_reset.argtypes = [ctypes.c_void_p]
        L.ob_model_forward.restype = ctypes.c_int
        L.ob_model_forward.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, _f32p]
        L.ob_generate.restype = ctypes.c_int
        L.ob_generate.argtypes = [ctypes.c_void_p, _i32p, ctypes.c_int, ctypes.c_int, _i32p,
                                  ctypes.POINTER(ctypes.c_int)]
        _lib = L
    return _lib


def _fp(a):
    return a.ctypes.data_as(_f32p)


def _bp(a):
    return a.ctypes.data_as(_u8p)


def set_threads(n: int) -> None:
    lib().ob_set_threads(int(n))


def get_threads() -> int:
    return lib().ob_get_threads()


def half_to_float(h: int) -> float:
    return lib().ob_half_to_float(h)


def float_to_half(f: float) -> int:
    return lib().ob_float_to_half(f)


def synth_fill(seed: int, tensor_id: int, start: int, n: int, std: float = 0.02) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().ob_synth_fill(seed, tensor_id, start, n, std, _fp(out))
    return out


def type_bytes(qtype: int, n: int) -> int:
    be, bb = TYPE_BLOCK[qtype]
    assert n % be == 0
    return n // be * bb


def quantize(qtype: int, x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32).ravel()
    out = np.empty(type_bytes(qtype, x.size), np.uint8)
    assert lib().ob_quantize(qtype, _fp(x), x.size, _bp(out)) == 0
    return out


def dequantize(qtype: int, data: np.ndarray, offset: int, n: int) -> np.ndarray:
    data = np.ascontiguousarray(data, np.uint8)
    out = np.empty(n, np.float32)
    assert lib().ob_dequantize(qtype, _bp(data), offset, n, _fp(out)) == 0
    return out


def synth_quantized(qtype: int, seed: int, tensor_id: int, n: int, std: float = 0.02) -> np.ndarray:
    out = np.empty(type_bytes(qtype, n), np.uint8)
    assert lib().ob_synth_quantized(qtype, seed, tensor_id, n, std, _bp(out)) == 0
    return out


def matvec(qtype: int, w: np.ndarray, woff: int, x: np.ndarray, K: int, N: int) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty(N, np.float32)
    assert lib().ob_matvec(qtype, _bp(np.ascontiguousarray(w, np.uint8)), woff, _fp(x), _fp(y), K, N) == 0
    return y


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    out = np.empty_like(x)
    lib().ob_rmsnorm(_fp(out), _fp(x), _fp(w), x.size, eps)
    return out


def softmax(x: np.ndarray) -> np.ndarray:
    v = np.array(x, np.float32)
    lib().ob_softmax(_fp(v), v.size)
    return v


def argmax(x: np.ndarray) -> int:
    x = np.ascontiguousarray(x, np.float32)
    return lib().ob_argmax(_fp(x), x.size)


def rope(q: np.ndarray, k: np.ndarray, n_heads: int, n_kv: int, hs: int, base: float, position: float,
         interleaved: bool):
    q = np.array(q, np.float32)
    k = np.array(k, np.float32)
    lib().ob_rope(_fp(q), _fp(k), n_heads, n_kv, hs, base, position, int(interleaved))
    return q, k


def glu(hb: np.ndarray, hb2: np.ndarray, gelu: bool) -> np.ndarray:
    h = np.array(hb, np.float32)
    h2 = np.ascontiguousarray(hb2, np.float32)
    lib().ob_glu(_fp(h), _fp(h2), h.size, int(gelu))
    return h


class OracleModel:
    """Synthetic model held by the oracle: same seed -> same packed bytes as
    the device generator (brew_model_synthesize)."""

    def __init__(self, cfg: ModelConfig, seed: int):
        self.cfg = cfg
        self._c = cfg.to_c()
        self.h = lib().ob_model_synth(ctypes.byref(self._c), seed)
        if not self.h:
            raise ValueError("oracle: unsupported model config")

    def close(self):
        if self.h:
            lib().ob_model_free(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def tensor(self, which: int) -> np.ndarray:
        n = ctypes.c_int64()
        p = lib().ob_model_tensor(self.h, which, ctypes.byref(n))
        if not p:
            return None
        return np.ctypeslib.as_array(ctypes.cast(p, _u8p), shape=(n.value,))

    def vector(self, which: int):
        n = ctypes.c_int64()
        p = lib().ob_model_vector(self.h, which, ctypes.byref(n))
        if not p or n.value == 0:
            return None
        return np.ctypeslib.as_array(ctypes.cast(p, _f32p), shape=(n.value,))

    def reset(self):
        lib().ob_model_reset(self.h)

    def forward(self, token: int, pos: int) -> np.ndarray:
        out = np.empty(self.cfg.vocab_size, np.float32)
        rc = lib().ob_model_forward(self.h, token, pos, _fp(out))
        if rc != 0:
            raise ValueError("oracle forward: bad token/pos")
        return out

    def generate(self, prompt, max_new: int) -> list:
        p = np.ascontiguousarray(prompt, np.int32)
        limit = max_new if max_new > 0 else self.cfg.seq_len
        out = np.zeros(max(limit, 1), np.int32)
        n = ctypes.c_int()
        rc = lib().ob_generate(self.h, p.ctypes.data_as(_i32p), p.size, max_new, out.ctypes.data_as(_i32p),
                               ctypes.byref(n))
        if rc == -2:
            raise RuntimeError("context full")
        if rc != 0:
            raise ValueError("oracle generate failed")
        return out[: n.value].tolist()
