"""Builds libt2sc.so in-tree (next to this file, under t2sc/) with nvcc for sm_100a.

Usage: python build.py [--force]. Called by __graft_entry__.build().
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "t2sc", "libt2sc.so")
SOURCES = ["api.cu", "hashmap.cu", "scan.cu", "conv_tc.cu", "conv_simt.cu", "convert.cu", "subdiv.cu", "selftest.cu", "norm.cu", "dist.cu", "block.cu", "pipeline.cu", "synth.cpp"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _stale():
    if not os.path.exists(OUT):
        return True
    t = os.path.getmtime(OUT)
    deps = [os.path.join(CSRC, f) for f in os.listdir(CSRC)]
    deps.append(os.path.join(HERE, "..", "include", "t2sc.h"))
    return any(os.path.getmtime(d) > t for d in deps)


def build(force=False, verbose=False):
    if not force and not _stale():
        return OUT
    nvcc = os.environ.get("NVCC", "nvcc")
    cmd = [nvcc, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3", "-shared",
           "--expt-relaxed-constexpr", "-o", OUT + ".tmp"]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    cmd += [os.path.join(CSRC, f) for f in SOURCES]
    cmd += ["-lpthread", "-ldl"]
    subprocess.run(cmd, check=True)
    os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
