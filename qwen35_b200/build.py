"""Build libq35b.so in-tree for sm_100a (nvcc cross-compiles without a GPU).

    python -m qwen35_b200.build          # or: python qwen35_b200/build.py
"""
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
SRC = os.path.join(PKG, "csrc")
LIB = os.path.join(PKG, "lib", "libq35b.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    # no multiply-add contraction: every product and sum rounds separately,
    # which is what the bit-exact paths (block folds, GDN recurrence) rely on
    "-fmad=false",
    "-Xcompiler", "-fPIC", "-shared", "-ldl",
]


def sources():
    return sorted(os.path.join(SRC, f) for f in os.listdir(SRC) if f.endswith((".cu", ".cuh")))


def up_to_date():
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    deps = sources() + [os.path.join(ROOT, "include", "q35.h"), os.path.abspath(__file__)]
    return all(os.path.getmtime(d) <= t for d in deps)


def build(force=False, verbose=False):
    if not force and up_to_date():
        return LIB
    os.makedirs(os.path.dirname(LIB), exist_ok=True)
    tmp = LIB + ".tmp"
    cmd = [NVCC] + FLAGS + ["-I", os.path.join(ROOT, "include"), "-o", tmp, os.path.join(SRC, "q35b.cu")]
    if verbose:
        print(" ".join(cmd))
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("nvcc failed building libq35b.so")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
