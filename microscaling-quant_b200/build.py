"""Build libmxq_b200.so, the C-ABI library of the mxq B200 kernels, in-tree (mxq/_lib/).

    python microscaling-quant_b200/build.py [--force] [--verbose]

Every .cu under csrc/ is compiled for sm_100a only (-gencode arch=compute_100a,code=sm_100a) with IEEE arithmetic
kept exact: no fused multiply-add contraction (--fmad=false), no flush-to-zero, IEEE division and square root.
Objects go to _build/ and are rebuilt when their source or any header is newer.
"""
import argparse
import glob
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB_DIR = os.path.join(HERE, "mxq", "_lib")
LIB = os.path.join(LIB_DIR, "libmxq_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "--extended-lambda", "-Xcompiler", "-fPIC", "--fmad=false",
         "-ftz=false", "-prec-div=true", "-prec-sqrt=true", "-I", os.path.join(ROOT, "include")]


def _headers():
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(ROOT, "include", "*.h"))


def _stale(obj, src, newest_header):
    return not os.path.exists(obj) or os.path.getmtime(obj) < max(os.path.getmtime(src), newest_header)


def build(force=False, verbose=False, ptxas_v=False):
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIB_DIR, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    newest = max([os.path.getmtime(h) for h in _headers()] + [0.0])
    jobs = []
    for src in sources:
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
        if force or _stale(obj, src, newest):
            cmd = [NVCC, *ARCH, *FLAGS, *(["-Xptxas", "-v"] if ptxas_v else []), "-c", src, "-o", obj]
            jobs.append((src, cmd))

    def run(job):
        src, cmd = job
        r = subprocess.run(cmd, capture_output=True, text=True)
        return src, r

    failed = []
    with ThreadPoolExecutor(max(1, min(len(jobs), os.cpu_count() or 1))) as ex:
        for src, r in ex.map(run, jobs):
            if verbose or r.returncode:
                sys.stderr.write(r.stdout + r.stderr)
            if r.returncode:
                failed.append(src)
    if failed:
        raise RuntimeError("nvcc failed: " + ", ".join(os.path.basename(f) for f in failed))
    objs = [os.path.join(BUILD, os.path.basename(s)[:-3] + ".o") for s in sources]
    if force or jobs or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        cmd = [NVCC, *ARCH, "-shared", "-o", LIB, *objs, "-lcudart"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError("link failed")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true", help="print registers / spills / shared memory per kernel")
    a = ap.parse_args()
    print(build(a.force, a.verbose, a.ptxas_v))
