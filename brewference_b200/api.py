"""Host-side mirror of the reference's hot-path interfaces over the C ABI.

Names and argument meaning follow the Java sources (paths relative to
src/main/java/com/epicmonstrosity/brewference/):

  PackedTensor          QuantizedWeights.Q8Block (gguf/QuantizedWeights.java:26-35),
                        holding the GGUF blocks unchanged in HBM
  Linear.matmul         transformer/math/Linear.java:40-65
  QuantizedWeights      gguf/QuantizedWeights.java:37-85 (dequantizeRow)
  DeviceModel.forward   TransformerGraph.forward (transformer/TransformerGraph.java:17)
  DeviceModel.generate  GenericModelSession.generate, greedy (runtime/ModelRunner.java:122-206)

Errors are the Java exception types: IllegalArgumentException,
IllegalStateException (see _native).
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

from . import _native as N
from .config import BrewConfig, ModelConfig, TYPE_BLOCK
from ._native import IllegalArgumentException, IllegalStateException  # noqa: F401


def _f32(a):
    return a.ctypes.data_as(N.c_f32p)


def _i32(a):
    return a.ctypes.data_as(N.c_i32p)


PREFILL_TOKENS, PREFILL_BATCHED = 0, 1   # brew_model_set_prefill modes


class PackedTensor:
    """A weight tensor of GGUF blocks resident in HBM (the device-side Q8Block)."""

    def __init__(self, handle: int, owned: bool = True):
        self.handle = handle
        self.owned = owned

    @classmethod
    def upload(cls, qtype: int, data: np.ndarray, n_elements: int) -> "PackedTensor":
        data = np.ascontiguousarray(data, np.uint8)
        be, bb = TYPE_BLOCK[qtype]
        if n_elements % be == 0 and data.size < n_elements // be * bb:
            raise IllegalArgumentException(N.ERR_INVALID_ARG, "fewer bytes than the tensor needs")
        h = ctypes.c_void_p()
        N.check(N.lib().brew_tensor_upload(qtype, data.ctypes.data, n_elements, ctypes.byref(h)), "upload")
        return cls(h.value)

    def info(self):
        t, n, nb = ctypes.c_int(), ctypes.c_int64(), ctypes.c_int64()
        N.check(N.lib().brew_tensor_info(self.handle, ctypes.byref(t), ctypes.byref(n), ctypes.byref(nb)))
        return t.value, n.value, nb.value

    @property
    def type(self) -> int:
        return self.info()[0]

    @property
    def n_elements(self) -> int:
        return self.info()[1]

    def read_bytes(self, offset: int = 0, n: int = None) -> np.ndarray:
        qt, total, _ = self.info()
        n = total - offset if n is None else n
        be, bb = TYPE_BLOCK[qt]
        out = np.empty(n // be * bb, np.uint8)
        N.check(N.lib().brew_tensor_read(self.handle, offset, n, out.ctypes.data), "tensor_read")
        return out

    def device_ptr(self) -> int:
        p = ctypes.c_void_p()
        N.check(N.lib().brew_tensor_device_ptr(self.handle, ctypes.byref(p)))
        return p.value

    def dequantize_row(self, offset: int, n: int) -> np.ndarray:
        out = np.empty(n, np.float32)
        N.check(N.lib().brew_dequantize_row(self.handle, offset, n, _f32(out)), "dequantize_row")
        return out

    def free(self):
        if self.handle and self.owned:
            N.lib().brew_tensor_free(self.handle)
        self.handle = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class Linear:
    """transformer/math/Linear.java"""

    @staticmethod
    def matmul(output: np.ndarray, input: np.ndarray, weights: PackedTensor, weights_offset: int, input_size: int,
               output_size: int) -> None:
        """output[r] = sum_k W[weights_offset + r*input_size + k] * input[k] (Linear.java:40-65)."""
        if weights is None or getattr(weights, "handle", None) is None:
            raise IllegalArgumentException(N.ERR_INVALID_ARG, "Weight block cannot be null")
        if input is None or output is None:
            raise IllegalArgumentException(N.ERR_INVALID_ARG, "Input and output arrays cannot be null")
        if output.dtype != np.float32 or input.dtype != np.float32 or not output.flags.c_contiguous:
            raise IllegalArgumentException(N.ERR_INVALID_ARG, "float32 contiguous arrays expected")
        if input.size < input_size or output.size < output_size:
            raise IllegalArgumentException(N.ERR_INVALID_ARG, "array shorter than its size argument")
        x = np.ascontiguousarray(input)
        N.check(N.lib().brew_matmul(_f32(output), _f32(x), weights.handle, weights_offset, input_size, output_size),
                "Linear.matmul")

    @staticmethod
    def prep_bytes(input_size: int, batch: int = 1) -> int:
        return int(N.lib().brew_prep_bytes(input_size, batch))

    @staticmethod
    def prepare_input_device(x_ptr: int, input_size: int, batch: int, prep_ptr: int, stream: int = 0) -> None:
        N.check(N.lib().brew_prepare_input_dev(x_ptr, input_size, batch, prep_ptr, stream or None), "prepare_input")

    @staticmethod
    def matmul_prepared_device(y_ptr: int, prep_ptr: int, weights: PackedTensor, weights_offset: int, input_size: int,
                               output_size: int, batch: int = 1, stream: int = 0) -> None:
        N.check(N.lib().brew_matmul_prepared_dev(y_ptr, prep_ptr, weights.handle, weights_offset, input_size,
                                                 output_size, batch, stream or None), "matmul_prepared")

    @staticmethod
    def matmul_device(y_ptr: int, x_ptr: int, weights: PackedTensor, weights_offset: int, input_size: int,
                      output_size: int, batch: int = 1, stream: int = 0) -> None:
        """Device-pointer, batched form (x [batch][input_size] -> y [batch][output_size])."""
        N.check(N.lib().brew_matmul_dev(y_ptr, x_ptr, weights.handle, weights_offset, input_size, output_size, batch,
                                        stream), "Linear.matmul_device")


class GemmPlan:
    """A Q8_0 / Q4_0 matrix repacked for the tcgen05 GEMM
    (brew_gemm_plan_*): run() multiplies T token vectors at once."""

    def __init__(self, weights: PackedTensor, weights_offset: int, input_size: int, output_size: int):
        h = ctypes.c_void_p()
        N.check(N.lib().brew_gemm_plan_create(weights.handle, weights_offset, input_size, output_size,
                                              ctypes.byref(h)), "gemm_plan_create")
        self.handle = h.value
        self.input_size, self.output_size = input_size, output_size

    def run(self, y_ptr: int, x_ptr: int, tokens: int, stream: int = 0) -> None:
        """y [tokens][output_size] = W x for x [tokens][input_size] (device pointers)."""
        N.check(N.lib().brew_gemm_plan_run(self.handle, y_ptr, x_ptr, tokens, stream or None), "gemm_plan_run")

    def free(self):
        if self.handle:
            N.lib().brew_gemm_plan_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def tp_rows(rows: int, nranks: int, rank: int):
    """Rows [r0, r1) of an N-row matrix that `rank` of `nranks` owns in the
    tensor-parallel forward."""
    r0, r1 = ctypes.c_int64(), ctypes.c_int64()
    N.check(N.lib().brew_tp_rows(rows, nranks, rank, ctypes.byref(r0), ctypes.byref(r1)), "tp_rows")
    return r0.value, r1.value


def comm_unique_id() -> bytes:
    """The 128-byte NCCL id rank 0 creates and shares (e.g. through
    torch.distributed's object broadcast)."""
    buf = ctypes.create_string_buffer(128)
    N.check(N.lib().brew_comm_unique_id(buf), "comm_unique_id")
    return buf.raw


class Communicator:
    """A NCCL communicator over the GPUs of one box (one process per GPU)."""

    def __init__(self, uid: bytes, nranks: int, rank: int):
        assert len(uid) == 128
        h = ctypes.c_void_p()
        N.check(N.lib().brew_comm_init(uid, nranks, rank, ctypes.byref(h)), "comm_init")
        self.handle, self.nranks, self.rank = h.value, nranks, rank

    def close(self):
        if self.handle:
            N.lib().brew_comm_free(self.handle)
            self.handle = None


class GgufFile:
    """A memory-mapped GGUF checkpoint (brew_gguf_open): the header, metadata
    and tensor infos as the reference's gguf/Reader.java reads them, and the
    model config as GgufConfigParser and the per-architecture loaders derive
    it.  Needs no GPU."""

    def __init__(self, path: str):
        h = ctypes.c_void_p()
        N.check(N.lib().brew_gguf_open(os.fsencode(path), ctypes.byref(h)), "gguf_open")
        self.handle = h.value
        self.path = path

    def config(self) -> ModelConfig:
        c = BrewConfig()
        N.check(N.lib().brew_gguf_config(self.handle, ctypes.byref(c)), "gguf_config")
        kw = {f: getattr(c, f) for f, _ in BrewConfig._fields_}
        return ModelConfig(name=os.path.basename(self.path), **kw)

    def tensors(self) -> list:
        """[(name, ggml type, elements, absolute file offset of the data)]"""
        n = ctypes.c_int64()
        N.check(N.lib().brew_gguf_tensor_count(self.handle, ctypes.byref(n)))
        out = []
        name = ctypes.create_string_buffer(512)
        t, ne, off = ctypes.c_int(), ctypes.c_int64(), ctypes.c_int64()
        for i in range(n.value):
            N.check(N.lib().brew_gguf_tensor_info(self.handle, i, name, len(name), ctypes.byref(t), ctypes.byref(ne),
                                                  ctypes.byref(off)))
            out.append((name.value.decode(), t.value, ne.value, off.value))
        return out

    def close(self):
        if self.handle:
            N.lib().brew_gguf_close(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()


class DeviceModel:
    """A device-resident model: weights, fp32 KV caches and the CUDA graphs of
    its forward pass."""

    def __init__(self, handle: int, cfg: ModelConfig, max_batch: int):
        self.handle = handle
        self.cfg = cfg
        self.max_batch = max_batch

    @classmethod
    def synthesize(cls, cfg: ModelConfig, seed: int, max_batch: int = 1) -> "DeviceModel":
        c = cfg.to_c()
        h = ctypes.c_void_p()
        N.check(N.lib().brew_model_synthesize(ctypes.byref(c), seed, max_batch, ctypes.byref(h)), "model_synthesize")
        return cls(h.value, cfg, max_batch)

    @classmethod
    def load_gguf(cls, path: str, max_batch: int = 1) -> "DeviceModel":
        """GgufCheckpointLoader.loadWeights + model creation in one call
        (brew_model_load_gguf): packed blocks from the file to HBM unchanged."""
        with GgufFile(path) as g:
            cfg = g.config()
        h = ctypes.c_void_p()
        N.check(N.lib().brew_model_load_gguf(os.fsencode(path), max_batch, ctypes.byref(h)), "model_load_gguf")
        return cls(h.value, cfg, max_batch)

    @classmethod
    def create(cls, cfg: ModelConfig, tensors: dict, vectors: dict, max_batch: int = 1) -> "DeviceModel":
        """tensors: name -> PackedTensor (token_embd, output, wq, wk, wv, wo, w_gate, w_up, w_down);
        vectors: name -> float32 arrays (rms_att, rms_ffn, rms_final, post_att, post_ffn, rms_q, rms_k,
        q_bias, k_bias, v_bias), concatenated over layers."""
        w = N.ModelWeights()
        keep = []
        for name in ("token_embd", "output", "wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down"):
            t = tensors.get(name)
            setattr(w, name, t.handle if t is not None else None)
        for name in ("rms_att", "rms_ffn", "rms_final", "post_att", "post_ffn", "rms_q", "rms_k", "q_bias", "k_bias",
                     "v_bias"):
            v = vectors.get(name)
            if v is not None:
                v = np.ascontiguousarray(v, np.float32)
                keep.append(v)
                setattr(w, name, _f32(v))
        c = cfg.to_c()
        h = ctypes.c_void_p()
        N.check(N.lib().brew_model_create(ctypes.byref(c), ctypes.byref(w), max_batch, ctypes.byref(h)), "model_create")
        m = cls(h.value, cfg, max_batch)
        m._tensors = tensors
        return m

    def tensor(self, which: int) -> PackedTensor:
        h = ctypes.c_void_p()
        N.check(N.lib().brew_model_tensor(self.handle, which, ctypes.byref(h)))
        return PackedTensor(h.value, owned=False)

    def forward(self, tokens, positions, want_logits: bool = True):
        """TransformerGraph.forward for len(tokens) sequences; returns
        (logits [batch][vocab] or None, argmax ids [batch])."""
        t = np.ascontiguousarray(np.atleast_1d(tokens), np.int32)
        p = np.ascontiguousarray(np.atleast_1d(positions), np.int32)
        b = t.size
        logits = np.empty((b, self.cfg.vocab_size), np.float32) if want_logits else None
        am = np.empty(b, np.int32)
        N.check(N.lib().brew_model_forward(self.handle, _i32(t), _i32(p), b, _f32(logits) if want_logits else None,
                                           _i32(am)), "forward")
        return logits, am

    def generate(self, prompt, max_new_tokens: int) -> list:
        """Greedy generation with the reference's token order."""
        pr = np.ascontiguousarray(prompt, np.int32)
        limit = max_new_tokens if max_new_tokens > 0 else self.cfg.seq_len
        out = np.zeros(max(limit, 1), np.int32)
        n = ctypes.c_int32()
        N.check(N.lib().brew_session_generate(self.handle, _i32(pr), pr.size, max_new_tokens, _i32(out),
                                              ctypes.byref(n)), "generate")
        return out[: n.value].tolist()

    def prefill(self, prompt, stream: int = 0) -> None:
        """GenericModelSession.prefill from a reset session."""
        pr = np.ascontiguousarray(prompt, np.int32)
        N.check(N.lib().brew_session_prefill(self.handle, _i32(pr), pr.size, stream or None), "prefill")

    def decode(self, n_steps: int, stream: int = 0, want_tokens: bool = True):
        """n greedy decode steps from the session state; returns the ids
        (synchronising) or None (enqueue only, on `stream`)."""
        out = np.empty(max(n_steps, 1), np.int32) if want_tokens else None
        N.check(N.lib().brew_session_decode(self.handle, n_steps, _i32(out) if want_tokens else None, stream or None),
                "decode")
        return out[:n_steps].tolist() if want_tokens else None

    def set_trace(self, on: bool = True) -> None:
        N.check(N.lib().brew_model_set_trace(self.handle, int(on)))

    def trace(self) -> list:
        """%globaltimer stamps (ns) of the last decode step, per CTA: start,
        then per phase: input landed, prep done, last weight stage in, work
        done, phase end."""
        buf = (ctypes.c_int64 * (1 << 18))()
        n = ctypes.c_int32()
        N.check(N.lib().brew_model_trace(self.handle, buf, 1 << 18, ctypes.byref(n)))
        return list(buf[: n.value])

    def step_kernels(self, batch: int = 1) -> int:
        n = ctypes.c_int32()
        N.check(N.lib().brew_model_step_kernels(self.handle, batch, ctypes.byref(n)))
        return n.value

    def reset(self):
        N.check(N.lib().brew_model_reset(self.handle), "reset")

    def set_prefill(self, mode: int) -> None:
        """How prefill / generate fill the KV cache with the prompt:
        PREFILL_TOKENS (token by token, the reference's order) or
        PREFILL_BATCHED (prompt chunks through each layer together, the
        matrices on the tcgen05 GEMM)."""
        N.check(N.lib().brew_model_set_prefill(self.handle, int(mode)), "set_prefill")

    def set_tp(self, comm: "Communicator") -> None:
        """Shards this model's matrices by rows over `comm` (every rank holds
        the same model); the forward then all-gathers each projection."""
        N.check(N.lib().brew_model_set_tp(self.handle, comm.handle), "set_tp")
        self.comm = comm

    def close(self):
        if self.handle:
            N.lib().brew_model_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
