"""Build the in-tree CUDA library ``ferret_b200/libferret_moe.so`` for sm_100a.

    python -m ferret_b200.build [--verbose] [--force]

Each ``csrc/*.cu`` is compiled by nvcc into ``_build/`` (in parallel) and the
objects are linked into one shared library with the CUDA runtime linked
statically, so the library loads on machines without a GPU driver (the
driver-API entry point the TMA descriptors need is resolved at run time
through the runtime).  ``kernel_result.cu`` becomes the benchmark binary
``ferret_b200/ferret_kernel_result`` linked against that library.
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
LIB = os.path.join(HERE, "libferret_moe.so")
BIN = os.path.join(HERE, "ferret_kernel_result")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CFLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
          "--expt-relaxed-constexpr", "-I", INCLUDE]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build ferret_b200")
    return cand


def _sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _deps():
    return [os.path.join(CSRC, f) for f in os.listdir(CSRC)] + [
        os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE)] + [
        os.path.join(HERE, "kernel_result.cu")]


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, force: bool = False, ptxas_verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = _sources()
    deps = _deps()
    if not force and not _stale(LIB, deps + [__file__]) and not _stale(BIN, deps + [__file__]):
        return LIB
    cc = nvcc()
    extra = ["-Xptxas", "-v"] if ptxas_verbose else []

    def compile_one(src):
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
        cmd = [cc, *ARCH, *CFLAGS, *extra, "-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
        return obj, r.stderr

    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        results = list(ex.map(compile_one, srcs))
    objs = [o for o, _ in results]
    if verbose or ptxas_verbose:
        for _, err in results:
            if err:
                print(err, file=sys.stderr)
    tmp = LIB + ".tmp"
    cmd = [cc, *ARCH, "-shared", "-Xcompiler", "-fPIC", "-cudart", "static", *objs, "-o", tmp]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    build_kernel_result(cc, verbose)
    return LIB


def build_kernel_result(cc: str, verbose: bool = False) -> str:
    """The self-contained benchmark binary (KERNEL_RESULT lines), linked
    against the library next to it."""
    src = os.path.join(HERE, "kernel_result.cu")
    cmd = [cc, *ARCH, "-O2", "-std=c++17", src, "-o", BIN, "-L", HERE, "-lferret_moe",
           "-Xlinker", "-rpath,$ORIGIN", "-cudart", "static"]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"kernel_result build failed:\n{r.stdout}\n{r.stderr}")
    return BIN


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas", action="store_true", help="print ptxas register/smem usage")
    a = ap.parse_args()
    print(build(verbose=a.verbose, force=a.force, ptxas_verbose=a.ptxas))


if __name__ == "__main__":
    main()
