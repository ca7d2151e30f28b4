"""Running the end-to-end harness (oracle/e2e_harness.c) from the tests.

oracle/_ref/e2e_ref is picolm with its own attention loops; oracle/_ref/e2e_pl
is the same program with model.c's attention blocks calling this module.
Both are built by `make -C oracle e2e` where the reference sources exist.
"""
import os
import subprocess

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
E2E_REF = os.path.join(ROOT, "oracle", "_ref", "e2e_ref")
E2E_PL = os.path.join(ROOT, "oracle", "_ref", "e2e_pl")


def have(binary: str) -> bool:
    return os.path.isfile(binary) and os.access(binary, os.X_OK)


def run(binary: str, gguf: str, n_prompt: int, n_gen: int, seed: int = 1, threads: int = 4,
        timeout: int = 1800):
    """(tokens, margins, summary dict) of one greedy run."""
    p = subprocess.run([binary, gguf, str(n_prompt), str(n_gen), str(seed), str(threads)],
                       capture_output=True, text=True, timeout=timeout)
    if p.returncode != 0:
        raise RuntimeError(f"{os.path.basename(binary)} failed ({p.returncode}):\n{p.stderr[-2000:]}")
    toks, margins, summary = [], [], {}
    for line in p.stdout.splitlines():
        f = line.split()
        if f and f[0] == "T":
            toks.append(int(f[2]))
            margins.append(float(f[3]))
        elif f and f[0] == "S":
            summary = {k: float(v) for k, v in (x.split("=") for x in f[1:])}
    return toks, margins, summary


def first_divergence(a, b):
    for i, (x, y) in enumerate(zip(a, b)):
        if x != y:
            return i
    return None if len(a) == len(b) else min(len(a), len(b))
