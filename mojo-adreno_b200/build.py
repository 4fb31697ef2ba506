"""Builds libmq.so (all CUDA sources, sm_100a) into the mq package directory, in-tree.

Usage: python build.py [--force]. Also called by __graft_entry__.build(). The library is one
translation unit (csrc/libmq.cu); it is rebuilt when any csrc/ or include/ file is newer.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
OUT = os.path.join(HERE, "mq", "libmq.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC,-O2,-fvisibility=hidden",
    "-shared", "--expt-relaxed-constexpr",
]


def _sources():
    files = []
    for d in (CSRC, INCLUDE):
        for root, _, names in os.walk(d):
            files += [os.path.join(root, n) for n in names if n.endswith((".cu", ".cuh", ".h", ".hpp"))]
    return files


def stale():
    if not os.path.exists(OUT):
        return True
    t = os.path.getmtime(OUT)
    return any(os.path.getmtime(f) > t for f in _sources())


def build(force=False, verbose=False):
    if not force and not stale():
        return OUT
    cmd = [NVCC, *FLAGS, "-I", INCLUDE, os.path.join(CSRC, "libmq.cu"), "-o", OUT + ".tmp"]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + " ".join(cmd) + "\n" + r.stdout + r.stderr)
    if verbose:
        sys.stderr.write(r.stderr)
    os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
