"""Build recipe for libllamacuda.so (sm_100a) -- in-tree, no JIT cache.

Compiles every CUDA / C++ source under csrc/ with nvcc for
`-gencode arch=compute_100a,code=sm_100a` and links one shared library with a
static CUDA runtime, so the .so travels with the source tree.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(BUILD, "libllamacuda.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
              "--expt-relaxed-constexpr", "-I", CSRC, "-I", INCLUDE]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found")
    return cand


def sources() -> list[str]:
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cpp")))


def _headers_mtime() -> float:
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hs.append(os.path.join(INCLUDE, "llamacuda.h"))
    return max(os.path.getmtime(h) for h in hs)


def build(verbose: bool = False, ptxas_verbose: bool = False, force: bool = False) -> str:
    """Compile csrc/ into _build/libllamacuda.so; returns the library path."""
    nvcc = _nvcc()
    objdir = os.path.join(BUILD, "obj")
    os.makedirs(objdir, exist_ok=True)
    hdr_t = _headers_mtime()
    jobs = []
    objs = []
    for src in sources():
        obj = os.path.join(objdir, os.path.basename(src) + ".o")
        objs.append(obj)
        fresh = os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(src), hdr_t)
        if fresh and not force:
            continue
        cmd = [nvcc, *ARCH, *NVCC_FLAGS, "-c", src, "-o", obj]
        if ptxas_verbose and src.endswith(".cu"):
            cmd += ["-Xptxas", "-v"]
        jobs.append(cmd)

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        return cmd, r

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        for cmd, r in ex.map(run, jobs):
            out = (r.stdout or "") + (r.stderr or "")
            if r.returncode != 0:
                raise RuntimeError(f"nvcc failed: {' '.join(cmd)}\n{out}")
            if out.strip() and (verbose or ptxas_verbose):
                print(out, file=sys.stderr)
    if jobs or not os.path.exists(LIB) or force:
        cmd = [nvcc, *ARCH, "-shared", "-cudart", "static", "-o", LIB, *objs, "-lpthread", "-ldl", "-lrt"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}{r.stderr}")
    return LIB


if __name__ == "__main__":
    build(verbose=True, ptxas_verbose="-v" in sys.argv, force="-f" in sys.argv)
    print(LIB)
