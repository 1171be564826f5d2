"""Build libcsaq_b200.so (the C-ABI library) in-tree for sm_100a.

    python csaq-quant_b200/build.py [--jobs N] [--clean]

Each .cu under csrc/ is compiled by nvcc to an object with
``-gencode arch=compute_100a,code=sm_100a -lineinfo -O3``; quant.cu, whose
results must be bit-exact with the reference's fp32 arithmetic, adds
``-fmad=false``. The objects are linked into csaq/lib/libcsaq_b200.so.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT_DIR = os.path.join(HERE, "csaq", "lib")
OBJ_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(OUT_DIR, "libcsaq_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3",
                 "-I", os.path.join(REPO, "include"), "-I", CSRC,
                 "--expt-relaxed-constexpr"]
PER_FILE = {"quant.cu": ["-fmad=false"]}


def sources():
    return sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))


def _compile(src: str, verbose: bool) -> str:
    obj = os.path.join(OBJ_DIR, src[:-3] + ".o")
    srcp = os.path.join(CSRC, src)
    deps = [srcp] + [os.path.join(CSRC, h) for h in os.listdir(CSRC) if h.endswith((".cuh", ".h"))]
    deps.append(os.path.join(REPO, "include", "csaq_b200.h"))
    if os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(d) for d in deps):
        return obj
    cmd = [NVCC] + COMMON + PER_FILE.get(src, []) + ["-c", srcp, "-o", obj]
    if verbose:
        print(" ".join(cmd))
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
    if r.stderr.strip() and verbose:
        print(r.stderr)
    return obj


def build(jobs: int = 0, verbose: bool = False) -> str:
    os.makedirs(OUT_DIR, exist_ok=True)
    os.makedirs(OBJ_DIR, exist_ok=True)
    srcs = sources()
    jobs = jobs or min(len(srcs), os.cpu_count() or 4)
    with cf.ThreadPoolExecutor(jobs) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), srcs))
    if os.path.exists(LIB) and os.path.getmtime(LIB) >= max(os.path.getmtime(o) for o in objs):
        return LIB
    cmd = [NVCC] + ARCH + ["-shared", "-o", LIB] + objs + ["-lcudart", "-lcuda"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--jobs", type=int, default=0)
    ap.add_argument("--clean", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    if a.clean and os.path.isdir(OBJ_DIR):
        for f in os.listdir(OBJ_DIR):
            os.remove(os.path.join(OBJ_DIR, f))
    print(build(a.jobs, a.verbose))
    sys.exit(0)
