"""Build libturboquant_b200.so in-tree with nvcc for sm_100a.

    python -m gemma4metal_b200.build [--force] [-v]

Each csrc/*.cu is compiled to an object under gemma4metal_b200/_build/ (not
committed), then linked into gemma4metal_b200/libturboquant_b200.so, which
ships to the GPU hosts next to the sources.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
OBJ = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libturboquant_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
              "-Xcompiler", "-fvisibility=hidden", "-I" + os.path.join(ROOT, "include"),
              "-Xptxas", "-warn-spills"]


def nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    inc = os.path.join(ROOT, "include")
    hs += [os.path.join(inc, f) for f in os.listdir(inc) if f.endswith((".h", ".hpp"))]
    return hs


CPP_TESTS = os.path.join(ROOT, "tests", "cpp")


def cpp_test_binary(name: str) -> str:
    """Path of the built C++ test program tests/cpp/<name>.cpp."""
    return os.path.join(OBJ, name + "_cpp")


def build_cpp_tests(verbose: bool = False) -> list:
    """Compile tests/cpp/*.cpp against the C++ API (include/turboquant.hpp) and
    the built library; binaries go to _build/ and find the library by rpath."""
    out = []
    if not os.path.isdir(CPP_TESTS):
        return out
    for f in sorted(os.listdir(CPP_TESTS)):
        if not f.endswith(".cpp"):
            continue
        src = os.path.join(CPP_TESTS, f)
        exe = cpp_test_binary(f[:-4])
        if os.path.exists(exe) and os.path.getmtime(exe) >= max(
                os.path.getmtime(src), os.path.getmtime(LIB), max(os.path.getmtime(h) for h in headers())):
            out.append(exe)
            continue
        cmd = [nvcc(), "-O2", "-std=c++17", "-I" + os.path.join(ROOT, "include"), src, "-o", exe,
               "-L" + PKG, "-lturboquant_b200", "-lcudart", "-Xlinker", "-rpath=" + PKG,
               "-Xlinker", "-rpath=$ORIGIN/.."]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"C++ test build failed for {src}:\n{r.stdout}\n{r.stderr}")
        out.append(exe)
    return out


def _compile(src: str, verbose: bool, ptxas_v: bool) -> str:
    obj = os.path.join(OBJ, os.path.basename(src)[:-3] + ".o")
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-c", src, "-o", obj]
    if ptxas_v:
        cmd += ["-Xptxas", "-v"]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    if ptxas_v or (verbose and r.stderr.strip()):
        print(r.stderr, file=sys.stderr)
    return obj


def build(force: bool = False, verbose: bool = False, ptxas_v: bool = False) -> str:
    os.makedirs(OBJ, exist_ok=True)
    srcs = sources()
    newest_hdr = max(os.path.getmtime(h) for h in headers())
    todo = []
    for s in srcs:
        obj = os.path.join(OBJ, os.path.basename(s)[:-3] + ".o")
        if force or ptxas_v or not os.path.exists(obj) or \
                os.path.getmtime(obj) < max(os.path.getmtime(s), newest_hdr):
            todo.append(s)
    if todo:
        with cf.ThreadPoolExecutor(max_workers=min(8, len(todo))) as ex:
            list(ex.map(lambda s: _compile(s, verbose, ptxas_v), todo))
    objs = [os.path.join(OBJ, os.path.basename(s)[:-3] + ".o") for s in srcs]
    if todo or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        cmd = [nvcc(), *ARCH, "-shared", "-o", LIB + ".tmp", *objs, "-lcudart"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        os.replace(LIB + ".tmp", LIB)
    build_cpp_tests(verbose)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv,
                ptxas_v="--ptxas" in sys.argv))
