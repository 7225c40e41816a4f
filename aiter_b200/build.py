"""Build the in-tree C-ABI library `aiter_b200/libaiter_b200.so` for sm_100a.

    python -m aiter_b200.build [--verbose]

Each .cu under aiter_b200/csrc is compiled by nvcc to an object in _build/ (in
parallel, skipped when up to date) and linked into one shared library.  The
library has no torch dependency; it links only the CUDA runtime.
"""
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(ROOT, "_build")
LIB = os.path.join(PKG, "libaiter_b200.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc():
    p = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(p):
        raise RuntimeError("nvcc not found")
    return p


def _flags(verbose):
    f = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-I" + os.path.join(ROOT, "include")] + ARCH
    if verbose:
        f += ["-Xptxas", "-v"]
    return f


def _headers():
    hs = [os.path.join(CSRC, h) for h in os.listdir(CSRC) if h.endswith((".cuh", ".h"))]
    hs.append(os.path.join(ROOT, "include", "aiter_b200.h"))
    return hs


def _compile(src, obj, verbose):
    cmd = [nvcc(), "-c", src, "-o", obj] + _flags(verbose)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    return r.stdout + r.stderr


def build(verbose=False, force=False):
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))
    hdr_mtime = max(os.path.getmtime(h) for h in _headers())
    jobs = []
    objs = []
    for s in srcs:
        o = os.path.join(BUILD, os.path.basename(s)[:-3] + ".o")
        objs.append(o)
        if force or verbose or not os.path.exists(o) or os.path.getmtime(o) < max(os.path.getmtime(s), hdr_mtime):
            jobs.append((s, o))
    logs = []
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(8, len(jobs))) as ex:
            for log in ex.map(lambda j: _compile(j[0], j[1], verbose), jobs):
                logs.append(log)
    if jobs or not os.path.exists(LIB):
        tmp = LIB + ".tmp"
        cmd = [nvcc(), "-shared", "-o", tmp] + objs + ARCH + ["-lcudart"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    if verbose:
        print("\n".join(logs))
    return LIB


if __name__ == "__main__":
    print(build(verbose="--verbose" in sys.argv, force="--force" in sys.argv))
