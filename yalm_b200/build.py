"""In-tree build of the native libraries.

  yalm_b200/libyalm_b200.so  — the decode engine (CUDA, sm_100a only) behind include/yalm_b200.h

Run `python -m yalm_b200.build` (or `__graft_entry__.build()`).  nvcc cross-compiles for sm_100a
without a GPU.  Objects go to yalm_b200/_build/; rebuilds are incremental on source timestamps.
"""
from __future__ import annotations

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libyalm_b200.so")

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-O3", "-I" + os.path.join(ROOT, "include"),
]
CU_SOURCES = ["gemv.cu", "attention.cu", "persistent.cu", "engine.cu", "capi.cu", "noalloc.cu", "sampler.cu", "loader.cu", "prefill_gemm.cu", "prefill.cu", "prefill_attn_tc.cu", "prefill_run.cu"]
HEADERS = ["common.cuh", "gemv.cuh", "attention.cuh", "persistent.cuh", "launch.h", "engine.h", "loader.h", "prefill.cuh",
           "prefill_gemm.cuh", "sampler.cuh", "tmap.h"]


def _newer(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd):
    r = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"command failed ({r.returncode}): {' '.join(cmd)}\n{r.stdout}")
    return r.stdout


def build_engine(verbose: bool = False, ptxas_info: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    hdrs = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(ROOT, "include", "yalm_b200.h")]
    objs = []
    jobs = []
    for src in CU_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src + ".o")
        objs.append(o)
        if _newer(o, [s] + hdrs) or ptxas_info:
            extra = ["-Xptxas", "-v"] if ptxas_info else []
            jobs.append([NVCC] + NVCC_FLAGS + extra + ["-c", s, "-o", o])
    if jobs:
        with ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            for out in ex.map(_run, jobs):
                if verbose or ptxas_info:
                    sys.stdout.write(out)
    if jobs or _newer(LIB, objs):
        _run([NVCC] + ARCH + ["-shared", "-o", LIB] + objs)
    return LIB


def build_all(verbose: bool = False) -> None:
    build_engine(verbose=verbose)


if __name__ == "__main__":
    build_engine(verbose=True, ptxas_info="--ptxas" in sys.argv)
    print(LIB)
