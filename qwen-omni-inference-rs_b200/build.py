"""Builds liblq8.so (the C-ABI library) in-tree for sm_100a with nvcc.

Usage: python qwen-omni-inference-rs_b200/build.py [--force]
The shared library lands next to this file, so it travels with the repository snapshot.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "liblq8.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

SOURCES = ["lq8_runtime.cu", "lq8_q8.cu", "lq8_gemv.cu", "lq8_gemm_tc.cu", "lq8_gemm_f16.cu", "lq8_attn_prefill.cu", "lq8_moe.cu", "lq8_comm.cu", "lq8_ops.cu", "lq8_attention.cu", "lq8_decode.cu", "lq8_sample.cu", "lq8_qwen3.cu"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-I", INCLUDE,
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _deps() -> list[str]:
    files = [os.path.join(CSRC, f) for f in os.listdir(CSRC)]
    files.append(os.path.join(INCLUDE, "lq8.h"))
    files.append(os.path.abspath(__file__))
    return files


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src: str, force: bool) -> str:
    obj = os.path.join(BUILD, os.path.splitext(src)[0] + ".o")
    if force or _stale(obj, _deps()):
        cmd = [_nvcc(), *NVCC_FLAGS, "-c", os.path.join(CSRC, src), "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stderr}")
    return obj


def build(force: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    if not force and not _stale(LIB, _deps()):
        return LIB
    with cf.ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        objs = list(ex.map(lambda s: _compile(s, force), SOURCES))
    tmp = LIB + ".tmp"
    cmd = [_nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", tmp, *objs,
           "-Xcompiler", "-fPIC"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
