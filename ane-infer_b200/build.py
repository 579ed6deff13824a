"""Build libab2.so (the CUDA kernels + C ABI) for sm_100a with nvcc, in-tree.

    python ane-infer_b200/build.py [--verbose-ptxas] [--jobs N]

Each csrc/*.cu is compiled to _build/*.o with
``-gencode arch=compute_100a,code=sm_100a -lineinfo -O3`` and linked into
ane-infer_b200/libab2.so with a static CUDA runtime. The command-line benchmark
ane-infer_b200/ab2_bench (ab2_bench.cpp, a plain C++ caller of the C ABI) is linked against
it. Targets are rebuilt only when a source or header is newer.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libab2.so")
CLI_SRC = os.path.join(HERE, "ab2_bench.cpp")
CLI = os.path.join(HERE, "ab2_bench")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC,-fvisibility=hidden",
         "-I", os.path.join(ROOT, "include"), "-I", CSRC]


def nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _headers():
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(ROOT, "include", "*.h"))


def _compile(src: str, ptxas_v: bool) -> str:
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    newest = max([os.path.getmtime(src)] + [os.path.getmtime(h) for h in _headers()])
    if os.path.exists(obj) and os.path.getmtime(obj) >= newest and not ptxas_v:
        return obj
    cmd = [nvcc(), *ARCH, *FLAGS, "-c", src, "-o", obj]
    if ptxas_v:
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{r.stderr}")
    if ptxas_v:
        sys.stderr.write(r.stderr)
    return obj


def build(verbose_ptxas: bool = False, jobs: int = 8) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose_ptxas), srcs))
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        cmd = [nvcc(), *ARCH, "-shared", "-o", LIB, *objs, "-cudart", "static", "-lpthread", "-ldl", "-lrt"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr}")
    build_cli()
    return LIB


def build_cli(out: str = CLI, lib_dir: str = HERE, lib: str = "ab2", extra: tuple = ()) -> str:
    """Compile ab2_bench.cpp with g++ and link it against lib{lib}.so in lib_dir; at run time
    the binary looks for the library in its own directory. `extra` adds sources."""
    header = os.path.join(ROOT, "include", "ab2.h")
    deps = [CLI_SRC, header, *extra]
    if os.path.exists(out) and os.path.getmtime(out) >= max(os.path.getmtime(d) for d in deps) and not extra:
        return out
    cmd = ["g++", "-O2", "-std=c++17", "-pthread", "-Wall", "-Wextra", "-I", os.path.join(ROOT, "include"), CLI_SRC, *extra,
           "-o", out]
    if lib:  # the library is looked up beside the binary first
        cmd += ["-L", lib_dir, f"-l{lib}", "-Wl,-rpath,$ORIGIN"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"g++ failed on {CLI_SRC}:\n{r.stderr}")
    return out


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose-ptxas", action="store_true")
    ap.add_argument("--jobs", type=int, default=8)
    a = ap.parse_args()
    print(build(a.verbose_ptxas, a.jobs))
