"""Build recipe for libtllm_kv.so (sm_100a) and the C++ facade test binary.

Compiles the CUDA kernels with nvcc for sm_100a only
(-gencode arch=compute_100a,code=sm_100a), the host manager and the C++
facade with g++, and links one shared library in-tree at
tiny-llm_b200/lib/libtllm_kv.so (static cudart, no libcuda link: the TMA
encoder is resolved through cudaGetDriverEntryPointByVersion at run time).
Objects go to tiny-llm_b200/_build/. Rebuilds only what changed.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB_DIR = PKG / "lib"
LIB = LIB_DIR / "libtllm_kv.so"
INCLUDE = ROOT / "include"
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")
CXX = shutil.which("g++") or "g++"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr"]
CXX_FLAGS = ["-O2", "-std=c++17", "-fPIC", "-Wall", "-Wextra", "-Wno-unused-parameter"]

CU_SOURCES = ["kv_append.cu", "paged_decode.cu", "paged_prefill_tc.cu", "qkv_append.cu", "qkv_append_tc.cu",
              "sampling.cu", "decode_static_scratch.cu"]
CPP_SOURCES = ["paged_kv.cpp"]
# The C++ facade (tiny_llm::KVCacheManager) is compiled by its user, with the
# user's include paths; the library itself exports only the C-ABI.
FACADE_SOURCE = CSRC / "kv_cache_manager.cpp"
HEADERS = ["kernels.h", "paged_kv.h", "ptx.cuh"]


def _run(cmd: list[str]) -> None:
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        sys.stderr.write(proc.stdout + proc.stderr)
        raise RuntimeError(f"build step failed: {' '.join(cmd)}")


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build_library(force: bool = False, verbose: bool = False) -> Path:
    """Compiles and links libtllm_kv.so; returns its path."""
    BUILD.mkdir(exist_ok=True)
    LIB_DIR.mkdir(exist_ok=True)
    common = [CSRC / h for h in HEADERS] + [INCLUDE / "tllm_kv.h", Path(__file__)]
    inc = [f"-I{INCLUDE}", f"-I{CSRC}", f"-I{CUDA_HOME / 'include'}"]
    objs = []
    for src in CU_SOURCES:
        s = CSRC / src
        o = BUILD / (src + ".o")
        if force or _stale(o, [s] + common):
            cmd = [NVCC, *ARCH, *NVCC_FLAGS, *inc, "-c", str(s), "-o", str(o)]
            if verbose:
                print(" ".join(cmd))
            _run(cmd)
        objs.append(o)
    for src in CPP_SOURCES:
        s = CSRC / src
        o = BUILD / (src + ".o")
        if force or _stale(o, [s] + common):
            cmd = [CXX, *CXX_FLAGS, *inc, "-c", str(s), "-o", str(o)]
            if verbose:
                print(" ".join(cmd))
            _run(cmd)
        objs.append(o)
    if force or _stale(LIB, objs):
        cmd = [NVCC, *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-cudart", "static"]
        if verbose:
            print(" ".join(cmd))
        _run(cmd)
    return LIB


def build_cpp_tests(force: bool = False) -> Path:
    """Builds tests/cpp/test_kv_cache_manager (ported reference KV tests)."""
    lib = build_library()
    src = ROOT / "tests" / "cpp" / "test_kv_cache_manager.cpp"
    out = BUILD / "test_kv_cache_manager"
    if force or _stale(out, [src, lib, FACADE_SOURCE, INCLUDE / "tiny_llm" / "kv_cache.h",
                             INCLUDE / "tllm_result.h"]):
        cmd = [CXX, "-O1", "-std=c++17", "-Wall", "-Wextra", "-Wno-unused-parameter", f"-I{INCLUDE}",
               f"-I{CUDA_HOME / 'include'}", str(src), str(FACADE_SOURCE),
               "-o", str(out), f"-L{LIB_DIR}", "-ltllm_kv", f"-Wl,-rpath,{LIB_DIR}",
               f"-L{CUDA_HOME / 'lib64'}", "-lcudart", f"-Wl,-rpath,{CUDA_HOME / 'lib64'}"]
        _run(cmd)
    return out


if __name__ == "__main__":
    print(build_library(force="--force" in sys.argv, verbose=True))
