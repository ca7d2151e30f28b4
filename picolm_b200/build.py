"""Build the sm_100a shared library picolm_b200/libpl_attn.so in tree.

    python -m picolm_b200.build            # or: make -C picolm_b200

nvcc compiles csrc/pl_attn.cu (which includes every kernel header) for
sm_100a only and links the CUDA runtime statically.  The driver API entry
point the module needs (cuTensorMapEncodeTiled) is looked up at run time
through cudaGetDriverEntryPoint, so the library has no link-time dependency
on libcuda and loads on a host without a GPU (its calls then fail with
PL_EDEVICE).  ptxas' resource report (registers, spills per kernel) is
kept beside the library in libpl_attn.resources.json, and the build fails if
the prefill kernels do not have the register count their warpgroup split
needs.
"""
from __future__ import annotations

import json
import os
import re
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


RESOURCES = os.path.join(HERE, "libpl_attn.resources.json")

# The prefill kernels split the registers of their launch allocation between
# warpgroups with setmaxnreg: they need exactly this many per thread at
# launch (65536 / 384 threads, rounded down to 8), or the increase of the
# softmax warpgroups can never be granted.
PREFILL_LAUNCH_REGS = 168


def parse_ptxas(text: str) -> dict:
    """{mangled kernel name: {"registers": n, "spill_stores": b, "spill_loads": b}}
    from nvcc -Xptxas=-v output."""
    out, cur = {}, None
    for line in text.splitlines():
        m = re.search(r"Compiling entry function '([^']+)'", line)
        if m:
            cur = m.group(1)
            out[cur] = {}
            continue
        if cur is None:
            continue
        m = re.search(r"(\d+) bytes spill stores, (\d+) bytes spill loads", line)
        if m:
            out[cur]["spill_stores"] = int(m.group(1))
            out[cur]["spill_loads"] = int(m.group(2))
        m = re.search(r"Used (\d+) registers", line)
        if m:
            out[cur]["registers"] = int(m.group(1))
    return out


def check_resources(res: dict) -> None:
    """Fail the build, not a later launch, when a toolkit change moves the
    prefill kernels off the register count their warpgroup split needs."""
    pf = {k: v for k, v in res.items() if "prefill_attn_kernel" in k}
    if not pf:
        raise RuntimeError("ptxas reported no prefill_attn_kernel")
    bad = {k: v.get("registers") for k, v in pf.items()
           if v.get("registers") != PREFILL_LAUNCH_REGS}
    if bad:
        raise RuntimeError(f"prefill kernels need {PREFILL_LAUNCH_REGS} registers per thread "
                           f"at launch, ptxas gave {bad}")


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date() and os.path.exists(RESOURCES):
        return OUT
    cmd = [nvcc(), "-Xptxas=-v", *NVCC_FLAGS, "-I", INCLUDE, "-o", OUT, SRC]
    if verbose:
        print(" ".join(cmd))
    r = subprocess.run(cmd, capture_output=True, text=True)
    if verbose or r.returncode:
        sys.stderr.write(r.stdout + r.stderr)
    if r.returncode:
        raise subprocess.CalledProcessError(r.returncode, cmd)
    res = parse_ptxas(r.stdout + r.stderr)
    with open(RESOURCES, "w") as f:
        json.dump(res, f, indent=1, sort_keys=True)
    check_resources(res)
    return OUT


if __name__ == "__main__":
    build(force=True, verbose="-v" in sys.argv)
    print(OUT)
