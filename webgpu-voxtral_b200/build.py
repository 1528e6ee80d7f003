"""Build libvoxtral_b200.so in-tree with nvcc for sm_100a (B200).

    python webgpu-voxtral_b200/build.py [--verbose]

The shared library is the C-ABI product (include/voxtral_b200.h).  It is built
in-tree so it travels with the repository snapshot to the GPU box.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIB = os.path.join(PKG, "libvoxtral_b200.so")
SOURCES = ["vx_engine.cu", "vx_noalloc.cu"]
DEPS = ["vx_engine.cu", "vx_noalloc.cu", "k_gemv.cuh", "k_attn.cuh", "k_misc.cuh", "k_step.cuh", "k_gemm.cuh", "k_codec.cuh",
        "vx_codec.cuh", "vx_common.cuh", "vx_rng.h"]


def nvcc() -> str:
    for c in (os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc"), shutil.which("nvcc")):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def flags(verbose: bool = False):
    f = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-lineinfo",
         "-Xcompiler", "-fPIC", "-Xcompiler", "-O3", "--expt-relaxed-constexpr",
         "-I", os.path.join(ROOT, "include"), "-I", CSRC]
    if verbose:
        f += ["-Xptxas", "-v"]
    return f


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, d) for d in DEPS] + [os.path.join(ROOT, "include", "voxtral_b200.h")]
    return all(os.path.getmtime(d) <= t for d in deps if os.path.exists(d))


def build(verbose: bool = False, force: bool = False) -> str:
    if not force and up_to_date():
        return LIB
    # The image exports CXX/CC pointing at a gcc without OpenMP; nvcc only needs a host compiler.
    env = dict(os.environ)
    host_cc = shutil.which("g++") or "g++"
    cmd = [nvcc(), *flags(verbose), "-ccbin", host_cc, "-shared", "-o", LIB + ".tmp",
           *[os.path.join(CSRC, s) for s in SOURCES], "-ldl"]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("nvcc failed")
    if verbose:
        sys.stderr.write(r.stderr)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    v = "--verbose" in sys.argv
    print(build(verbose=v, force=True))
