"""Builds ``libmeshb200.so`` (sm_100a) in-tree with nvcc.

Usage: ``python -m grokking_abmod_b200.build`` (or ``build()`` from Python).
The library exports the C ABI declared in ``include/meshb200.h``.
"""

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libmeshb200.so")

SOURCES = ["gpt_model.cu", "mesh_ops.cu", "gemm_tc.cu", "simple_model.cu", "config.cpp", "data.cpp",
           "simple_config.cpp", "checkpoint.cpp"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc():
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if cand and (os.path.sep not in cand or os.path.exists(cand)):
            return cand
    raise RuntimeError("nvcc not found")


def _stale():
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, f) for f in os.listdir(CSRC)]
    deps.append(os.path.join(ROOT, "include", "meshb200.h"))
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    """Compiles the library if any source is newer than it; returns its path."""
    if not force and not _stale():
        return LIB
    tmp = LIB + ".tmp"
    cmd = [_nvcc(), "-std=c++17", "-O3", "-lineinfo", "--threads", "0", *ARCH, "-shared", "-Xcompiler",
           "-fPIC,-ffp-contract=off",
           "-I", os.path.join(ROOT, "include"), "-o", tmp]
    cmd += [os.path.join(CSRC, s) for s in SOURCES]
    cmd += ["-ldl"]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + res.stdout + res.stderr)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
