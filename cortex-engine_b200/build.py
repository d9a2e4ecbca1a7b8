"""Build libcortex_b200.so (sm_100a) in-tree with nvcc.

    python cortex-engine_b200/build.py [--force] [--jobs N]

Each csrc/*.cu is compiled with relocatable device code (the per-device status
word is shared across files), then device-linked into one shared library at
cortex-engine_b200/cortex/libcortex_b200.so, next to the Python package that
loads it. Objects go to cortex-engine_b200/_build/ (git-ignored).
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(HERE, "_build")
OUT = os.path.join(HERE, "cortex", "libcortex_b200.so")

SOURCES = [
    "status.cu",
    "pack.cu",
    "tokenizer.cu",
    "dequant.cu",
    "norm.cu",
    "gemm_tc.cu",
    "gemm_simt.cu",
    "attention_tc.cu",
    "attention_ws.cu",
    "attention_simt.cu",
    "capi.cu",
    "head.cu",
    "forward.cu",
    "noalloc.cu",
    "batch.cpp",
    "ingest.cu",
    "rows.cu",
    "runner.cpp",
    "trace.cpp",
]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CFLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "-rdc=true", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
    "-I", INCLUDE, "-I", CSRC,
]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found")
    return cand


def _deps_mtime() -> float:
    paths = [os.path.join(CSRC, f) for f in os.listdir(CSRC)]
    paths.append(os.path.join(INCLUDE, "cortex_b200.h"))
    return max(os.path.getmtime(p) for p in paths)


# Host-only sources (.cpp) go to the host compiler directly.
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
HOST_CFLAGS = ["-O3", "-std=c++17", "-fPIC", "-Wall", "-I", INCLUDE, "-I", CSRC,
               "-I", os.path.join(CUDA_HOME, "include")]


def _compile(src: str, force: bool, extra: list[str]) -> str:
    obj = os.path.join(BUILD, os.path.splitext(src)[0] + ".o")
    srcp = os.path.join(CSRC, src)
    if (not force and os.path.exists(obj)
            and os.path.getmtime(obj) >= max(os.path.getmtime(srcp), _deps_mtime())):
        return obj
    if src.endswith(".cpp"):
        cmd = [shutil.which("g++") or "g++"] + HOST_CFLAGS + ["-c", srcp, "-o", obj]
    else:
        cmd = [nvcc()] + CFLAGS + extra + ["-c", srcp, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    if r.stderr.strip():
        sys.stderr.write(r.stderr)
    return obj


def build(force: bool = False, jobs: int | None = None, verbose_ptxas: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    extra = ["-Xptxas", "-v"] if verbose_ptxas else []
    jobs = jobs or min(len(SOURCES), os.cpu_count() or 4)
    with ThreadPoolExecutor(max_workers=jobs) as ex:
        objs = list(ex.map(lambda s: _compile(s, force, extra), SOURCES))
    if (not force and os.path.exists(OUT)
            and os.path.getmtime(OUT) >= max(os.path.getmtime(o) for o in objs)):
        return OUT
    cmd = [nvcc()] + ARCH + ["-shared", "-rdc=true", "-Xcompiler", "-fPIC"] + objs + ["-o", OUT]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("--ptxas-v", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, jobs=args.jobs, verbose_ptxas=args.ptxas_v))
