"""Build step for libct_b200.so (and the test harness libraries that link it).

The library is one CUDA translation unit compiled for sm_100a only
(`-gencode arch=compute_100a,code=sm_100a`: the tcgen05 / TMA instructions are
accepted only for the arch-specific target).  The CUDA runtime is linked
statically; the driver entry point for tensor-map encoding is resolved at run
time, so the .so needs only libcuda.so on the GPU host.
"""
from __future__ import annotations

import glob
import os
import subprocess

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
LIB = os.path.join(PKG_DIR, "libct_b200.so")
NVCC = os.environ.get("NVCC", "nvcc")
NVCC_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-lineinfo",
              "-Xcompiler", "-fPIC", "-shared"]


def _newer(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build_lib(force: bool = False, verbose: bool = False) -> str:
    deps = glob.glob(os.path.join(CSRC, "*")) + glob.glob(os.path.join(REPO_DIR, "include", "*.h"))
    if force or _newer(LIB, deps):
        cmd = [NVCC] + NVCC_FLAGS + ["-o", LIB, os.path.join(CSRC, "ct_b200.cu")]
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
    return LIB


def build_dropin_harness(reference_dir: str | None) -> str | None:
    """tests/bin/libref_decode_b200.so: the reference's model.h (from the
    reference tree) driven by oracle/ref_harness.c and linked against
    libct_b200.so -- the unmodified reference caller on this backend."""
    if not reference_dir or not os.path.exists(os.path.join(reference_dir, "model.h")):
        return None
    out_dir = os.path.join(REPO_DIR, "tests", "bin")
    os.makedirs(out_dir, exist_ok=True)
    out = os.path.join(out_dir, "libref_decode_b200.so")
    src = os.path.join(REPO_DIR, "oracle", "ref_harness.c")
    if _newer(out, [src, LIB]):
        subprocess.run(["gcc", "-O2", "-fPIC", "-shared", "-DBACKEND_CUDA", "-Wno-unused-function",
                        "-Wno-unused-variable", f"-I{reference_dir}", "-o", out, src, f"-L{PKG_DIR}", "-lct_b200",
                        "-Wl,-rpath,$ORIGIN/../../cohere-transcribe_b200", "-lpthread", "-lm"], check=True)
    return out


if __name__ == "__main__":
    build_lib(force=True, verbose=True)
