"""Build the sm_100a shared library in-tree: nvcc for the .cu files, g++ for the host
planner, objects under ``_build/``, the library next to this file.

    python llm-inference-server_b200/build.py [--force]

No GPU is needed (nvcc cross-compiles for sm_100a).  The library links the CUDA runtime
statically and reaches the driver only through the runtime's entry-point query, so it
loads on any machine with a CUDA 12.8+ driver.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB_NAME = "libpaged_attn_b200.so"
LIB = PKG / LIB_NAME

CU_SOURCES = ["api.cu", "decode_splitk.cu", "decode_mma.cu", "prefill_tc.cu", "prefill_persist.cu", "prefill_pair.cu", "attention_generic.cu", "kv_append.cu",
              "attention_noalloc.cu",
              "block_copy.cu", "peer_allreduce.cu", "oproj_allreduce.cu"]
CXX_SOURCES = ["step_plan.cpp"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; the CUDA toolkit is required to build the extension")


def _inputs() -> list[Path]:
    return [*(CSRC / s for s in CU_SOURCES + CXX_SOURCES), *CSRC.glob("*.h"), *CSRC.glob("*.cuh"),
            *(ROOT / "include").glob("*.h"), Path(__file__)]


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in _inputs())


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return LIB
    nvcc = _nvcc()
    cuda_home = Path(nvcc).resolve().parent.parent
    BUILD.mkdir(exist_ok=True)
    inc = ["-I", str(ROOT / "include"), "-I", str(CSRC)]
    jobs = []
    for s in CU_SOURCES:
        obj = BUILD / (s + ".o")
        jobs.append([nvcc, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
                     "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills", *inc, "-c", str(CSRC / s),
                     "-o", str(obj)])
    for s in CXX_SOURCES:
        obj = BUILD / (s + ".o")
        jobs.append(["g++", "-O3", "-fPIC", "-std=c++17", "-Wall", *inc, "-I", str(cuda_home / "include"),
                     "-c", str(CSRC / s), "-o", str(obj)])

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"build failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        return r.stderr

    with ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as ex:
        for err in ex.map(run, jobs):
            if verbose and err.strip():
                print(err, file=sys.stderr)
    objs = [str(BUILD / (s + ".o")) for s in CU_SOURCES + CXX_SOURCES]
    tmp = LIB.with_suffix(".so.tmp")
    run([nvcc, *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *objs])
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
