"""Build libcsaq_b200.so (the C-ABI library) in-tree for sm_100a.

    python csaq-quant_b200/build.py [--jobs N] [--clean] [--checked]

Each .cu under csrc/ is compiled by nvcc to an object with
``-gencode arch=compute_100a,code=sm_100a -lineinfo -O3``; quant.cu, whose
results must be bit-exact with the reference's fp32 arithmetic, adds
``-fmad=false``. The objects are linked into csaq/lib/libcsaq_b200.so.

--checked builds the same sources with -DCSAQ_CHECKED into
csaq/lib/libcsaq_b200_checked.so: kernels test the indices they take from
caller data (output rows, cache positions) and record failures instead of
touching memory out of range (csaq_guard_report). CSAQ_LIB=checked in the
environment makes csaq load it.
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
LIB_CHECKED = os.path.join(OUT_DIR, "libcsaq_b200_checked.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3",
                 "-I", os.path.join(REPO, "include"), "-I", CSRC,
                 "--expt-relaxed-constexpr"]
PER_FILE = {"quant.cu": ["-fmad=false"]}


def sources():
    return sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))


def _compile(src: str, verbose: bool, checked: bool = False) -> str:
    obj = os.path.join(OBJ_DIR, ("checked_" if checked else "") + src[:-3] + ".o")
    srcp = os.path.join(CSRC, src)
    deps = [srcp] + [os.path.join(CSRC, h) for h in os.listdir(CSRC) if h.endswith((".cuh", ".h"))]
    deps.append(os.path.join(REPO, "include", "csaq_b200.h"))
    if os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(d) for d in deps):
        return obj
    cmd = [NVCC] + COMMON + PER_FILE.get(src, []) + (["-DCSAQ_CHECKED"] if checked else []) + ["-c", srcp, "-o", obj]
    if verbose:
        print(" ".join(cmd))
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
    if r.stderr.strip() and verbose:
        print(r.stderr)
    return obj


def build(jobs: int = 0, verbose: bool = False, checked: bool = False) -> str:
    os.makedirs(OUT_DIR, exist_ok=True)
    os.makedirs(OBJ_DIR, exist_ok=True)
    srcs = sources()
    lib = LIB_CHECKED if checked else LIB
    jobs = jobs or min(len(srcs), os.cpu_count() or 4)
    with cf.ThreadPoolExecutor(jobs) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose, checked), srcs))
    if os.path.exists(lib) and os.path.getmtime(lib) >= max(os.path.getmtime(o) for o in objs):
        return lib
    cmd = [NVCC] + ARCH + ["-shared", "-o", lib] + objs + ["-lcudart", "-lcuda"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return lib


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--jobs", type=int, default=0)
    ap.add_argument("--clean", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--checked", action="store_true", help="build libcsaq_b200_checked.so (index guards)")
    a = ap.parse_args()
    if a.clean and os.path.isdir(OBJ_DIR):
        for f in os.listdir(OBJ_DIR):
            os.remove(os.path.join(OBJ_DIR, f))
    print(build(a.jobs, a.verbose, a.checked))
    sys.exit(0)
