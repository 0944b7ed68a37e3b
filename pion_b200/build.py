"""Build recipe for libpion_vector_b200.so (sm_100a only).

Every ``.cu`` file under ``pion_b200/csrc`` is compiled with nvcc for
``arch=compute_100a,code=sm_100a``, and every ``.cpp`` file (host-only code: the
HNSW graph builder) with the host C++ compiler, into ``pion_b200/_build/``; both are
linked into
``pion_b200/libpion_vector_b200.so`` (in-tree, so the library ships with the
repository snapshot).  The CUDA runtime is linked statically; the driver API is
reached through ``cudaGetDriverEntryPoint`` so no ``-lcuda`` is needed.

Usage: ``python -m pion_b200.build [--force] [--jobs N]``.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libpion_vector_b200.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O2,-Wall",
              "-Xptxas", "-warn-spills", "--expt-relaxed-constexpr", "-I", INCLUDE]


# Host-only sources: the HNSW builder's distance loops use AVX2 + FMA (the library
# checks the CPU before calling into them).
CXX_FLAGS = ["-O3", "-std=c++17", "-fPIC", "-Wall", "-mavx2", "-mfma", "-pthread"]


def cxx() -> str:
    for cand in (os.environ.get("CXX"), shutil.which("g++"), shutil.which("c++")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("no host C++ compiler found")


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the B200 library cannot be built")


def _sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cpp")))


def _headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hs += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]
    return hs


def _newest(paths):
    return max((os.path.getmtime(p) for p in paths), default=0.0)


def _compile(src: str, force: bool) -> str:
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    if not force and os.path.exists(obj) and os.path.getmtime(obj) >= max(
            os.path.getmtime(src), _newest(_headers())):
        return obj
    if src.endswith(".cpp"):
        cmd = [cxx(), *CXX_FLAGS, "-c", src, "-o", obj]
    else:
        cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compile failed on {os.path.basename(src)}:\n{r.stdout}\n{r.stderr}")
    return obj


def build(force: bool = False, jobs: int | None = None, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = _sources()
    jobs = jobs or min(len(srcs), os.cpu_count() or 1)
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        objs = list(ex.map(lambda s: _compile(s, force), srcs))
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < _newest(objs):
        cmd = [nvcc(), *ARCH, "-shared", "-o", LIB, *objs, "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    if verbose:
        print(LIB)
    return LIB


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    a = ap.parse_args(argv)
    build(force=a.force, jobs=a.jobs, verbose=True)


if __name__ == "__main__":
    sys.exit(main())
