"""Compile the native library and tools in-tree for sm_100a.

Outputs (git-ignored, shipped with the tree):
  gustann_b200/_lib/libgann.so   C ABI of include/gann.h
  gustann_b200/_lib/search_mem   CLI with the reference driver's flags
  gustann_b200/_lib/check_recall recall of a result file against an ivecs ground truth

Run ``python -m gustann_b200.build`` (idempotent; rebuilds when a source is newer).
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "_lib")
INCLUDE = os.path.join(ROOT, "include")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
LIB = os.path.join(OUT, "libgann.so")
CLI = os.path.join(OUT, "search_mem")
CHECK = os.path.join(OUT, "check_recall")

LIB_SOURCES = ["gann_search.cu", "gann_api.cu", "gann_loader.cpp", "gann_exact.cu", "gann_build.cu"]
HEADERS = ["gann_internal.hpp"]


def _newer(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd: list[str]) -> None:
    print("+", " ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


def build_lib(force: bool = False, verbose_ptxas: bool = False) -> str:
    os.makedirs(OUT, exist_ok=True)
    srcs = [os.path.join(CSRC, s) for s in LIB_SOURCES]
    deps = srcs + [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(INCLUDE, "gann.h")]
    if force or _newer(LIB, deps):
        cmd = [NVCC, *ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC,-O3",
               "-shared", "-I", INCLUDE, "-I", CSRC, *srcs, "-o", LIB + ".tmp", "-lpthread"]
        if verbose_ptxas:
            cmd.insert(1, "-Xptxas=-v")
        _run(cmd)
        os.replace(LIB + ".tmp", LIB)
    return LIB


def build_cli(force: bool = False) -> str:
    src = os.path.join(CSRC, "search_mem.cpp")
    deps = [src, LIB, os.path.join(INCLUDE, "gustann.hpp"), os.path.join(INCLUDE, "gann.h")]
    if force or _newer(CLI, deps):
        _run(["g++", "-O2", "-std=c++17", "-I", INCLUDE, src, "-o", CLI + ".tmp",
              "-L", OUT, "-lgann", "-Wl,-rpath,$ORIGIN"])
        os.replace(CLI + ".tmp", CLI)
    return CLI


def build_check(force: bool = False) -> str:
    src = os.path.join(CSRC, "check_recall.cpp")
    if force or _newer(CHECK, [src]):
        _run(["g++", "-O2", "-std=c++17", src, "-o", CHECK + ".tmp"])
        os.replace(CHECK + ".tmp", CHECK)
    return CHECK


def build_all(force: bool = False) -> None:
    build_lib(force)
    build_cli(force)
    build_check(force)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv)
