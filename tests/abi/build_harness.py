"""Compiles tests/abi/abi_harness.cpp against libenvgemm.so (g++, rpath to the in-tree library)."""
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
LIBDIR = os.path.join(ROOT, "invision_b200", "lib")


def build(out_dir):
    exe = os.path.join(out_dir, "abi_harness")
    subprocess.check_call(["g++", "-std=c++17", "-O2", "-I", os.path.join(ROOT, "include"),
                           os.path.join(HERE, "abi_harness.cpp"), "-L", LIBDIR, "-lenvgemm",
                           f"-Wl,-rpath,{LIBDIR}", "-o", exe])
    return exe
