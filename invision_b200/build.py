"""Builds libenvgemm.so in-tree for sm_100a (nvcc cross-compiles; no GPU needed)."""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = [os.path.join(HERE, "csrc", "envgemm.cu")]
INCLUDE = os.path.join(os.path.dirname(HERE), "include")


def deps():
    """Every source and header the library is compiled from."""
    csrc = os.path.join(HERE, "csrc")
    files = [os.path.join(csrc, f) for f in os.listdir(csrc) if f.endswith((".cu", ".cuh", ".hpp", ".h"))]
    return files + [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith((".h", ".hpp"))]
OUT = os.path.join(HERE, "lib", "libenvgemm.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
         "-Xcompiler", "-fPIC,-O3", "-shared"]


def needs_build():
    if not os.path.exists(OUT):
        return True
    t = os.path.getmtime(OUT)
    return any(os.path.getmtime(p) > t for p in deps())


def build(force=False, verbose=True):
    if not force and not needs_build():
        return OUT
    os.makedirs(os.path.dirname(OUT), exist_ok=True)
    cmd = [NVCC] + FLAGS + SRC + ["-o", OUT]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.check_call(cmd)
    return OUT


if __name__ == "__main__":
    build(force="--force" in sys.argv)
