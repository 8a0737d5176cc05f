"""Builds libcfi_b200.so (sm_100a kernels + the C ABI) in-tree with nvcc and g++.

Usage: python build.py [--force].  Objects go to _build/ beside this file; the library to
lib/libcfi_b200.so.  Every .cu file is compiled for sm_100a only (`-gencode
arch=compute_100a,code=sm_100a`); host C++ is compiled by g++ with contraction off so the
probe's host checks keep their operation order.
"""
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "lib", "libcfi_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
CXX = os.environ.get("CFI_CXX", "/usr/bin/g++")
CUDA_INC = "/usr/local/cuda/include"
NVFLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-O3", "-std=c++17",
           "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr",
           "-Xptxas", "-warn-spills"]
CXXFLAGS = ["-O2", "-std=c++17", "-fPIC", "-fvisibility=hidden", "-ffp-contract=off", "-Wall",
            "-I", CUDA_INC]


def _deps(src):
    deps = [src] + [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".hpp", ".cuh"))]
    deps.append(os.path.join(HERE, "..", "include", "cfi_subst.h"))
    deps.append(os.path.join(HERE, "..", "include", "cfi_cublas.h"))
    return [d for d in deps if os.path.exists(d)]


def _stale(out, deps):
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src, force):
    name = os.path.basename(src)
    out = os.path.join(OBJ, name + ".o")
    if not force and not _stale(out, _deps(src)):
        return out
    if src.endswith(".cu"):
        cmd = [NVCC] + NVFLAGS + ["-c", src, "-o", out]
    else:
        cmd = [CXX] + CXXFLAGS + ["-c", src, "-o", out]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("compile failed: %s\n%s%s" % (" ".join(cmd), r.stdout, r.stderr))
    return out


def build(force=False):
    os.makedirs(OBJ, exist_ok=True)
    os.makedirs(os.path.dirname(LIB), exist_ok=True)
    srcs = sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cpp")))
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(s, force), srcs))
    if force or _stale(LIB, objs):
        cmd = [NVCC, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-o", LIB] + objs + [
            "-Xcompiler", "-fPIC", "-lcudart_static", "-ldl", "-lpthread", "-lrt"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed: %s\n%s%s" % (" ".join(cmd), r.stdout, r.stderr))
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
