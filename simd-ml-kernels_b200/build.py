"""build.py — compile the B200 library in place.

  simd_ml_kernels/libsmk_cuda.so   the C ABI (include/smk_cuda.h) and every
                                   sm_100a kernel (csrc/*.cu), nvcc
                                   -gencode arch=compute_100a,code=sm_100a
  simd_ml_kernels/_core*.so        the Python module (csrc/core_pybind.cpp,
                                   pybind11), linked to libsmk_cuda.so

Runs without a GPU (nvcc cross-compiles). Incremental: an output is rebuilt
when a source or header it depends on is newer. `python build.py --force`
rebuilds everything. No -use_fast_math: the x and weight quantizers must
round exactly as the reference's IEEE arithmetic does.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
PKG = os.path.join(HERE, "simd_ml_kernels")
BUILD = os.path.join(HERE, "_build")
INCLUDE = os.path.join(REPO, "include")

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
CUDA_HOME = os.path.dirname(os.path.dirname(NVCC))
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
              "--expt-relaxed-constexpr", "-I" + INCLUDE] + ARCH
CU_SOURCES = ["gemv_quant.cu", "gemv_dense.cu", "gemv_dense_mma.cu", "gemv_int8.cu", "dequant.cu", "decode.cu",
              "smk_api.cu", "gemv_noalloc.cu"]
HEADERS = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))

LIB = os.path.join(PKG, "libsmk_cuda.so")
EXT_SUFFIX = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
CORE = os.path.join(PKG, "_core" + EXT_SUFFIX)


def _stale(out: str, deps: list[str]) -> bool:
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
        raise SystemExit(f"build failed: {os.path.basename(cmd[-1]) if cmd else ''}")


def _compile_cu(src: str, force: bool) -> str:
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    if force or _stale(obj, [src] + HEADERS):
        _run([NVCC] + NVCC_FLAGS + ["-c", src, "-o", obj])
    return obj


def build(force: bool = False, verbose: bool = True) -> None:
    os.makedirs(BUILD, exist_ok=True)
    srcs = [os.path.join(CSRC, s) for s in CU_SOURCES]
    with cf.ThreadPoolExecutor(max_workers=len(srcs)) as ex:
        objs = list(ex.map(lambda s: _compile_cu(s, force), srcs))
    if force or _stale(LIB, objs):
        _run([NVCC] + ARCH + ["-shared", "-o", LIB] + objs + ["-lcudart_static", "-lrt", "-ldl", "-lpthread"])
        if verbose:
            print(f"built {os.path.relpath(LIB, REPO)}")
    core_src = os.path.join(CSRC, "core_pybind.cpp")
    if force or _stale(CORE, [core_src, LIB] + HEADERS):
        import pybind11

        cxx = os.environ.get("SMK_CXX", "g++")
        _run([cxx, "-O2", "-std=c++17", "-shared", "-fPIC", "-Wall", "-fvisibility=hidden",
              "-I" + pybind11.get_include(), "-I" + sysconfig.get_paths()["include"], "-I" + INCLUDE,
              core_src, "-o", CORE, "-L" + PKG, "-lsmk_cuda", "-Wl,-rpath,$ORIGIN"])
        if verbose:
            print(f"built {os.path.relpath(CORE, REPO)}")


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    build(force=ap.parse_args().force)
