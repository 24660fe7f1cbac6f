"""brewference_b200 — B200 (sm_100a) implementation of brewference's
quantized-matmul hot path behind a C ABI (include/brew.h).

The native library (libbrew.so, built in-tree by brewference_b200/build.py)
is loaded on first use; every compute entry point raises if it is missing or
if no CUDA device is visible.  There is no CPU fallback.
"""
from .config import ModelConfig, PRESETS  # noqa: F401

__version__ = "0.1.0"
