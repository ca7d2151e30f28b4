"""Running the end-to-end harness (oracle/e2e_harness.c) from the tests.

oracle/_ref/e2e_ref is picolm with its own attention loops; oracle/_ref/e2e_pl
is the same program with model.c's attention blocks calling this module, and
oracle/_ref/e2e_blk the program whose whole attention sub-blocks (RMSNorm,
projections, attention, residual) call it.
Both are built by `make -C oracle e2e` where the reference sources exist.
"""
import os
import subprocess

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
E2E_REF = os.path.join(ROOT, "oracle", "_ref", "e2e_ref")
E2E_PL = os.path.join(ROOT, "oracle", "_ref", "e2e_pl")
E2E_BLK = os.path.join(ROOT, "oracle", "_ref", "e2e_blk")


def have(binary: str) -> bool:
    return os.path.isfile(binary) and os.access(binary, os.X_OK)


def run(binary: str, gguf: str, n_prompt: int, n_gen: int, seed: int = 1, threads: int = 4,
        timeout: int = 1800, save: str | None = None, load: str | None = None):
    """(tokens, margins, summary dict) of one greedy run; `save` / `load`
    name KVCP files for picolm's kvcache_save / kvcache_load."""
    cmd = [binary, gguf, str(n_prompt), str(n_gen), str(seed), str(threads)]
    if save:
        cmd += ["--save", save]
    if load:
        cmd += ["--load", load]
    p = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout)
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


def read_kvcp(path: str):
    """picolm's KVCP file (model.c:1144-1156): header (magic, n_pos, n_layers,
    kv_dim) and the K and V rows as [n_layers][n_pos][kv_dim] FP16 words."""
    import numpy as np
    raw = np.fromfile(path, np.uint8)
    head = raw[:16].view(np.uint32)
    n_pos, n_layers, kv_dim = (int(x) for x in head[1:4])
    body = raw[16:].view(np.uint16)
    n = n_layers * n_pos * kv_dim
    assert body.size == 2 * n, (body.size, n)
    return head, body[:n].reshape(n_layers, n_pos, kv_dim), body[n:].reshape(n_layers, n_pos, kv_dim)
