"""ctypes binding of libbrew.so (the C ABI declared in include/brew.h).

The library is loaded from this package directory on first use.  A missing
library raises NativeLibraryMissing: there is no Python or CPU fallback for
any compute entry point.
"""
from __future__ import annotations

import ctypes
import os
import re

from .config import BrewConfig

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("BREW_LIB") or os.path.join(HERE, "libbrew.so")   # BREW_LIB: another build of the library
HEADER = os.path.join(os.path.dirname(HERE), "include", "brew.h")

OK, ERR_INVALID_ARG, ERR_OUT_OF_BOUNDS, ERR_CUDA, ERR_NCCL, ERR_TIMEOUT, ERR_CONTEXT_FULL, ERR_UNSUPPORTED, \
    ERR_IO, ERR_NO_DEVICE = 0, -1, -2, -3, -4, -5, -6, -7, -8, -9


class NativeLibraryMissing(RuntimeError):
    pass


class BrewError(RuntimeError):
    """Base of the mapped C-ABI errors; `code` is the BREW_ERR_* value."""

    def __init__(self, code: int, msg: str):
        super().__init__(msg)
        self.code = code


class IllegalArgumentException(BrewError, ValueError):
    """Linear.validateMatmulArguments / bad arguments (Java IllegalArgumentException)."""


class IllegalStateException(BrewError):
    """Scale index out of bounds, context exhausted, device failure (Java IllegalStateException)."""


class IOExceptionError(BrewError, OSError):
    """Malformed tensor data (Java IOException in GgufWeightsLoader)."""


class NoDeviceError(BrewError):
    """No CUDA device is visible."""


def _exc_for(code: int):
    if code == ERR_INVALID_ARG:
        return IllegalArgumentException
    if code == ERR_IO:
        return IOExceptionError
    if code == ERR_NO_DEVICE:
        return NoDeviceError
    return IllegalStateException


_lib = None

c_f32p = ctypes.POINTER(ctypes.c_float)
c_i32p = ctypes.POINTER(ctypes.c_int32)
c_void_pp = ctypes.POINTER(ctypes.c_void_p)


class ModelWeights(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in ("token_embd", "output", "wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down")] + \
               [(n, c_f32p) for n in ("rms_att", "rms_ffn", "rms_final", "post_att", "post_ffn", "rms_q", "rms_k",
                                      "q_bias", "k_bias", "v_bias")]


def lib():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise NativeLibraryMissing(f"{LIB_PATH} is not built: run `python -m brewference_b200.build`")
    L = ctypes.CDLL(LIB_PATH)
    I, I64, V, S = ctypes.c_int, ctypes.c_int64, ctypes.c_void_p, ctypes.c_size_t
    sig = {
        "brew_last_error": (I, [ctypes.c_char_p, S]),
        "brew_init": (I, [I]),
        "brew_version": (ctypes.c_char_p, []),
        "brew_kernel_launches": (I64, []),
        "brew_type_bytes": (I64, [I, I64]),
        "brew_type_block": (I, [I, ctypes.POINTER(I), ctypes.POINTER(I)]),
        "brew_tensor_upload": (I, [I, V, I64, c_void_pp]),
        "brew_tensor_alloc": (I, [I, I64, c_void_pp]),
        "brew_tensor_write": (I, [V, I64, V, I64]),
        "brew_tensor_free": (I, [V]),
        "brew_tensor_info": (I, [V, ctypes.POINTER(I), ctypes.POINTER(I64), ctypes.POINTER(I64)]),
        "brew_tensor_device_ptr": (I, [V, c_void_pp]),
        "brew_tensor_read": (I, [V, I64, I64, V]),
        "brew_dequantize_row": (I, [V, I64, I64, c_f32p]),
        "brew_dequantize_row_dev": (I, [V, I64, I64, V, V]),
        "brew_matmul": (I, [c_f32p, c_f32p, V, I64, ctypes.c_int32, ctypes.c_int32]),
        "brew_matmul_dev": (I, [V, V, V, I64, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, V]),
        "brew_gemm_q8_dev": (I, [V, V, V, I64, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, V]),
        "brew_gemm_plan_create": (I, [V, I64, ctypes.c_int32, ctypes.c_int32, ctypes.POINTER(V)]),
        "brew_gemm_plan_run": (I, [V, V, V, ctypes.c_int32, V]),
        "brew_gemm_plan_free": (I, [V]),
        "brew_tp_rows": (I, [I64, ctypes.c_int32, ctypes.c_int32, ctypes.POINTER(I64), ctypes.POINTER(I64)]),
        "brew_comm_unique_id": (I, [ctypes.c_char_p]),
        "brew_comm_init": (I, [ctypes.c_char_p, ctypes.c_int32, ctypes.c_int32, ctypes.POINTER(V)]),
        "brew_comm_free": (I, [V]),
        "brew_model_set_tp": (I, [V, V]),
        "brew_model_set_prefill": (I, [V, ctypes.c_int32]),
        "brew_matmul_dev_static": (I, [V, V, V, I64, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, V]),
        "brew_model_create": (I, [ctypes.POINTER(BrewConfig), ctypes.POINTER(ModelWeights), ctypes.c_int32, c_void_pp]),
        "brew_model_synthesize": (I, [ctypes.POINTER(BrewConfig), ctypes.c_uint64, ctypes.c_int32, c_void_pp]),
        "brew_model_free": (I, [V]),
        "brew_model_config": (I, [V, ctypes.POINTER(BrewConfig)]),
        "brew_model_tensor": (I, [V, I, c_void_pp]),
        "brew_model_forward": (I, [V, c_i32p, c_i32p, ctypes.c_int32, c_f32p, c_i32p]),
        "brew_model_forward_dev": (I, [V, V, V, ctypes.c_int32, V, V, V]),
        "brew_session_generate": (I, [V, c_i32p, ctypes.c_int32, ctypes.c_int32, c_i32p, c_i32p]),
        "brew_model_reset": (I, [V]),
        "brew_session_prefill": (I, [V, c_i32p, ctypes.c_int32, V]),
        "brew_session_decode": (I, [V, ctypes.c_int32, c_i32p, V]),
        "brew_model_step_kernels": (I, [V, ctypes.c_int32, c_i32p]),
        "brew_model_set_trace": (I, [V, ctypes.c_int32]),
        "brew_model_trace": (I, [V, ctypes.POINTER(ctypes.c_int64), ctypes.c_int32, c_i32p]),
        "brew_gguf_open": (I, [ctypes.c_char_p, c_void_pp]),
        "brew_gguf_close": (I, [V]),
        "brew_gguf_config": (I, [V, ctypes.POINTER(BrewConfig)]),
        "brew_gguf_tensor_count": (I, [V, ctypes.POINTER(I64)]),
        "brew_gguf_tensor_info": (I, [V, I64, ctypes.c_char_p, S, ctypes.POINTER(I), ctypes.POINTER(I64),
                                      ctypes.POINTER(I64)]),
        "brew_model_load_gguf": (I, [ctypes.c_char_p, ctypes.c_int32, c_void_pp]),
        "brew_selftest_wait_timeout": (I, [I64, c_i32p]),
        "brew_prep_bytes": (I64, [ctypes.c_int32, ctypes.c_int32]),
        "brew_prepare_input_dev": (I, [V, ctypes.c_int32, ctypes.c_int32, V, V]),
        "brew_matmul_prepared_dev": (I, [V, V, V, I64, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, V]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def last_error() -> str:
    buf = ctypes.create_string_buffer(2048)
    lib().brew_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(rc: int, what: str = "") -> None:
    if rc != OK:
        msg = last_error()
        raise _exc_for(rc)(rc, f"{what}: {msg}" if what else msg)


def header_symbols() -> list:
    """Names of the functions include/brew.h declares."""
    with open(HEADER) as f:
        text = f.read()
    return sorted(set(re.findall(r"BREW_API\s+[\w\s\*]+?\b(brew_\w+)\s*\(", text)))


def init(device: int = -1) -> None:
    check(lib().brew_init(device), "brew_init")


def kernel_launches() -> int:
    return int(lib().brew_kernel_launches())
