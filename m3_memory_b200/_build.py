"""Builds libm3gpu.so (CUDA kernels + engine + C ABI, sm_100a) and the pybind
module ``_m3_async`` in-tree, next to this file.

Objects go to ``_build/`` at the repository root and are rebuilt only when a
source or header is newer.  Run ``python -m m3_memory_b200._build``.
"""
from __future__ import annotations

import os
import subprocess
import sys
import sysconfig
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
BUILD = ROOT / "_build"
LIB = PKG / "libm3gpu.so"

CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              *ARCH, f"-I{INCLUDE}", f"-I{CSRC}"]

CU_SOURCES = ["k_coarse.cu", "k_scan.cu", "k_scan_tc.cu", "k_kmeans.cu", "k_gemm_tc.cu",
              "engine.cu", "noalloc.cu"]
CPP_SOURCES = ["api.cpp", "faiss_io.cpp"]
HEADERS = ["common.cuh", "score.cuh", "topk.cuh", "tc.cuh", "kernels.h", "kernels_kmeans.h",
           "engine.h"]


def _newer(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(Path(d).stat().st_mtime > t for d in deps)


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(" ".join(map(str, cmd)) + "\n" + r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {cmd[0]} {cmd[-1]}")
    return r


def pybind_module_path() -> Path:
    suffix = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    return PKG / f"_m3_async{suffix}"


def build(verbose: bool = False) -> None:
    BUILD.mkdir(exist_ok=True)
    headers = [CSRC / h for h in HEADERS] + [INCLUDE / "m3gpu.h"]
    objs = []
    for src in CU_SOURCES + CPP_SOURCES:
        s = CSRC / src
        o = BUILD / (s.stem + ".o")
        objs.append(o)
        if _newer(o, [s, *headers]):
            cmd = [NVCC, *NVCC_FLAGS, "-c", str(s), "-o", str(o)]
            if src.endswith(".cpp"):
                cmd = [NVCC, "-x", "c++", *NVCC_FLAGS, "-c", str(s), "-o", str(o)]
            if verbose:
                print(" ".join(cmd))
            _run(cmd)
    if _newer(LIB, objs):
        _run([NVCC, *ARCH, "-shared", "-o", str(LIB), *map(str, objs)])
    mod = pybind_module_path()
    bsrc = CSRC / "bindings.cpp"
    if _newer(mod, [bsrc, INCLUDE / "m3gpu.h", LIB]):
        import pybind11

        py_inc = sysconfig.get_paths()["include"]
        _run(["g++", "-O2", "-std=c++17", "-shared", "-fPIC", "-fvisibility=hidden",
              f"-I{pybind11.get_include()}", f"-I{py_inc}", f"-I{INCLUDE}", str(bsrc),
              f"-L{PKG}", "-lm3gpu", "-Wl,-rpath,$ORIGIN", "-o", str(mod)])


if __name__ == "__main__":
    build(verbose="-v" in sys.argv)
    print(LIB)
    print(pybind_module_path())
