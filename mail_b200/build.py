"""Builds libmoe_b200.so (the C-ABI library) in-tree with nvcc for sm_100a.

Usage: python -m mail_b200.build [--verbose]   (or mail_b200.build.build())
The library has no torch dependency: it links the CUDA runtime statically and
reaches the driver API (cuTensorMapEncodeTiled) through cudaGetDriverEntryPoint.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD_DIR = os.path.join(HERE, "_build")
LIB_NAME = "libmoe_b200.so"
LIB_PATH = os.path.join(HERE, LIB_NAME)
SOURCES = ["moe_route.cu", "moe_rows.cu", "moe_prep.cu", "moe_gemm.cu", "moe_api.cu", "moe_ep.cu"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden"]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libmoe_b200.so")
    return cand


def _newer(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return False
    t = os.path.getmtime(target)
    return all(os.path.getmtime(d) <= t for d in deps)


def _headers() -> list[str]:
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hs.append(os.path.join(os.path.dirname(HERE), "include", "moe_b200.h"))
    return hs


def build(verbose: bool = False, force: bool = False, extra_flags: list[str] | None = None) -> str:
    """Compiles every source for sm_100a and links LIB_PATH; returns its path."""
    os.makedirs(BUILD_DIR, exist_ok=True)
    nvcc = _nvcc()
    headers = _headers()
    flags = COMMON_FLAGS + ARCH_FLAGS + (extra_flags or [])
    if verbose:
        flags = flags + ["-Xptxas", "-v"]

    def compile_one(src: str) -> str:
        path = os.path.join(CSRC, src)
        obj = os.path.join(BUILD_DIR, src.replace(".cu", ".o"))
        if not force and _newer(obj, [path] + headers):
            return obj
        cmd = [nvcc, *flags, "-c", path, "-o", obj]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{res.stdout}\n{res.stderr}")
        if verbose and (res.stdout or res.stderr):
            sys.stderr.write(res.stdout + res.stderr)
        return obj

    with ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        objs = list(ex.map(compile_one, SOURCES))
    if force or not _newer(LIB_PATH, objs):
        cmd = [nvcc, *ARCH_FLAGS, "-shared", "-Xcompiler", "-fPIC", *objs, "-o", LIB_PATH]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    return LIB_PATH


if __name__ == "__main__":
    print(build(verbose="--verbose" in sys.argv, force="--force" in sys.argv))
