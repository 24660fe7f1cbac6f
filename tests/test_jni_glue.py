"""The JNI glue (brewference_b200/csrc/jni/brew_jni.cpp) compiled, linked
against libbrew.so and run on the CPU.  No JDK exists in this image, so the
JNI types and JNIEnv functions come from a test-only header
(tests/jni_stub/jni.h) and a fake environment (tests/jni_stub/fake_env.cpp)
that records the exceptions the glue throws.  Checked: the glue builds with
-Wall -Werror, and the C-ABI errors become the Java exceptions the reference
throws for the same conditions (Linear.java:67-74 IllegalArgumentException,
GgufWeightsLoader / Reader IOException, IllegalStateException otherwise)."""
import os
import shutil
import subprocess

import pytest

from brewference_b200 import _native as N

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_jni_glue_builds_and_maps_errors(tmp_path):
    cxx = shutil.which("g++")
    if cxx is None:
        pytest.skip("no C++ compiler")
    lib = N.lib()._name
    exe = str(tmp_path / "jni_harness")
    subprocess.check_call([cxx, "-std=c++17", "-O1", "-Wall", "-Werror", "-I", os.path.join(ROOT, "tests", "jni_stub"),
                           "-I", os.path.join(ROOT, "include"),
                           os.path.join(ROOT, "brewference_b200", "csrc", "jni", "brew_jni.cpp"),
                           os.path.join(ROOT, "tests", "jni_stub", "fake_env.cpp"), lib,
                           "-Wl,-rpath," + os.path.dirname(lib), "-o", exe])
    bad = tmp_path / "not_a_checkpoint.gguf"
    bad.write_bytes(b"NOTGGUF" + bytes(64))
    out = subprocess.run([exe, str(bad)], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stderr
    lines = dict(l.split(": ", 1) for l in out.stdout.strip().splitlines())
    assert lines["matmul_null_weights"] == "java/lang/IllegalArgumentException | Weight block cannot be null"
    assert lines["matmul_null_arrays"].startswith("java/lang/IllegalArgumentException |")
    assert lines["load_gguf_bad_file"].startswith("java/io/IOException | Not a GGUF file")
    import torch
    if not torch.cuda.is_available():
        assert lines["init"].startswith("java/lang/IllegalStateException | no CUDA device")
