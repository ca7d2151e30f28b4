"""Build the sm_100a shared library picolm_b200/libpl_attn.so in tree.

    python -m picolm_b200.build            # or: make -C picolm_b200

nvcc compiles csrc/pl_attn.cu (which includes every kernel header) for
sm_100a only and links the CUDA runtime statically.  The driver API entry
point the module needs (cuTensorMapEncodeTiled) is looked up at run time
through cudaGetDriverEntryPoint, so the library has no link-time dependency
on libcuda and loads on a host without a GPU (its calls then fail with
PL_EDEVICE).
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "csrc", "pl_attn.cu")
OUT = os.path.join(HERE, "libpl_attn.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC,-O2", "-shared",
    "-cudart", "static",
    "--expt-relaxed-constexpr",
]


def nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources():
    csrc = os.path.join(HERE, "csrc")
    out = [os.path.join(csrc, f) for f in sorted(os.listdir(csrc))]
    out.append(os.path.join(INCLUDE, "pl_attn.h"))
    return out


def up_to_date() -> bool:
    if not os.path.exists(OUT):
        return False
    t = os.path.getmtime(OUT)
    return all(os.path.getmtime(s) <= t for s in sources())


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return OUT
    cmd = [nvcc(), *NVCC_FLAGS, "-I", INCLUDE, "-o", OUT, SRC]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    return OUT


if __name__ == "__main__":
    build(force=True, verbose="-v" in sys.argv)
    print(OUT)
