"""Build libvla_simd_b200.so in-tree (nvcc for sm_100a, g++ for host C++).

The library is one CUDA translation unit (csrc/kernels.cu) plus the host
runtime and the extern "C" boundary, linked with the static CUDA runtime so the
.so carries no dependency beyond the driver. Incremental: an object is rebuilt
when its source or any header in csrc/ is newer.

    python -m vla_simd_b200.build            # or: python vla_simd_b200/build.py
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libvla_simd_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
                     "-Xptxas", "-warn-spills"]
CXX_FLAGS = ["-std=c++17", "-O2", "-fPIC", "-fvisibility=hidden", "-Wall", "-Wno-unused-function"]

CUDA_SOURCES = ["kernels.cu", "no_alloc.cu"]
CXX_SOURCES = ["act_policy.cpp", "conv_exec.cpp", "dp_policy.cpp", "octo_policy.cpp", "t5_tokenizer.cpp", "smolvla_policy.cpp",
               "bpe_tokenizer.cpp",
               "host_quant.cpp", "model_files.cpp", "capi.cpp"]


def _cuda_home() -> str:
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    return os.path.dirname(os.path.dirname(os.path.realpath(nvcc)))


def _newest_header() -> float:
    t = 0.0
    for name in os.listdir(CSRC):
        if name.endswith((".h", ".cuh", ".cu")):
            t = max(t, os.path.getmtime(os.path.join(CSRC, name)))
    for name in os.listdir(os.path.join(ROOT, "include")):
        t = max(t, os.path.getmtime(os.path.join(ROOT, "include", name)))
    return t


def _compile(src: str, dep_time: float) -> str:
    out = os.path.join(OBJ, os.path.splitext(src)[0] + ".o")
    path = os.path.join(CSRC, src)
    if os.path.exists(out) and os.path.getmtime(out) >= max(os.path.getmtime(path), dep_time):
        return out
    cuda_inc = os.path.join(_cuda_home(), "include")
    if src.endswith(".cu"):
        cmd = ["nvcc", *NVCC_FLAGS, "-c", path, "-o", out]
    else:
        cmd = ["g++", *CXX_FLAGS, "-I" + cuda_inc, "-c", path, "-o", out]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return out


def build(verbose: bool = False) -> str:
    os.makedirs(OBJ, exist_ok=True)
    dep = _newest_header()
    with ThreadPoolExecutor(max_workers=4) as ex:
        objs = list(ex.map(lambda s: _compile(s, dep), CUDA_SOURCES + CXX_SOURCES))
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        # -Bsymbolic: the library's own calls bind to its own definitions, so a
        # process that also loads the reference's library (which exports the
        # same model ABI names) cannot redirect them
        cmd = ["nvcc", *ARCH, "-shared", "-cudart", "static", "-Xlinker", "-Bsymbolic", "-o", LIB, *objs, "-lcuda"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            # libcuda.so is only needed for the driver entry point query at
            # runtime; link without it if the stub is absent
            cmd = cmd[:-1]
            r = subprocess.run(cmd, capture_output=True, text=True)
            if r.returncode != 0:
                raise RuntimeError(f"link failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    if verbose:
        print(LIB)
    return LIB


if __name__ == "__main__":
    build(verbose=True)
    sys.exit(0)
