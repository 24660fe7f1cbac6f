"""Builds libbrew.so in-tree (brewference_b200/libbrew.so) for sm_100a.

    python -m brewference_b200.build [--force] [--jobs N]

Each .cu file under csrc/ is compiled with nvcc for
`-gencode arch=compute_100a,code=sm_100a` and linked into one shared
library with the static CUDA runtime.  The JNI glue (csrc/jni/) is added
only when a JDK's jni.h is found (JAVA_HOME).
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libbrew.so")
ROOT = os.path.dirname(HERE)

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
              "--expt-relaxed-constexpr", "-I", os.path.join(ROOT, "include")]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def sources() -> list:
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def headers() -> list:
    out = [os.path.join(ROOT, "include", "brew.h")]
    out += [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    return out


def _stale(target: str, deps: list) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src: str, verbose: bool) -> str:
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    if _stale(obj, [src] + headers()):
        cmd = [nvcc()] + ARCH + NVCC_FLAGS + ["-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.check_call(cmd)
    return obj


def build(force: bool = False, jobs: int = 0, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sources()
    if force:
        for f in os.listdir(BUILD):
            os.remove(os.path.join(BUILD, f))
    jobs = jobs or min(len(srcs), os.cpu_count() or 4)
    with cf.ThreadPoolExecutor(jobs) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), srcs))
    extra = []
    java_home = os.environ.get("JAVA_HOME", "")
    jni_src = os.path.join(CSRC, "jni", "brew_jni.cpp")
    if java_home and os.path.exists(os.path.join(java_home, "include", "jni.h")) and os.path.exists(jni_src):
        jobj = os.path.join(BUILD, "brew_jni.o")
        subprocess.check_call(["g++", "-O2", "-fPIC", "-std=c++17", "-I", os.path.join(java_home, "include"),
                               "-I", os.path.join(java_home, "include", "linux"), "-I", os.path.join(ROOT, "include"),
                               "-c", jni_src, "-o", jobj])
        extra.append(jobj)
    if force or _stale(LIB, objs + extra):
        cmd = [nvcc()] + ARCH + ["-shared", "-o", LIB] + objs + extra + ["-lcuda"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.check_call(cmd)
    return LIB


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=0)
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args(argv)
    print(build(a.force, a.jobs, a.verbose))


if __name__ == "__main__":
    sys.exit(main())
