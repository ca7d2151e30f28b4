"""Random-init LLaMA-architecture model in GGUF v3 with Q4_K weights.

Test infrastructure for the end-to-end check (config 2): picolm loads the
file with its own parser (model.c:286-527) and runs greedy decoding once on
the CPU and once with attention through the B200 module.

* GGUF v3 container: header, metadata key/values, tensor infos, data
  aligned to 32 bytes; the metadata keys are the `llama.*` keys that
  picolm's parse_gguf reads (model.c:321-400).
* Q4_K blocks as picolm decodes them (quant.c:82-126, block_q4_K in
  quant.h:65-72): 256 weights = 8 sub-blocks of 32; sub-block j decodes as
  d*sc_j*q - dmin*mn_j with 6-bit sc_j, mn_j packed into 12 bytes and 4-bit
  q (two sub-blocks share a byte run, low nibble first).  The encoder here
  is our own: per sub-block an asymmetric [min(x,0), max(x)] range over 15
  steps, per super-block d and dmin = the largest step / offset over 63.
* Weights ~N(0, 0.02) from numpy's PCG64 with the given seed, tensor by
  tensor in file order; RMSNorm weights are 1.0 (F32).

Usage: python oracle/make_gguf.py OUT.gguf [--layers 22 --dim 2048 --ffn 5632
       --heads 32 --kv-heads 4 --vocab 32000 --ctx 2048 --seed 1]
"""
from __future__ import annotations

import argparse
import struct

import numpy as np

GGUF_MAGIC = 0x46554747
T_UINT32, T_FLOAT32, T_STRING = 4, 6, 8
TYPE_F32, TYPE_Q4_K = 0, 12
ALIGN = 32


def q4k_encode(w: np.ndarray, chunk_blocks: int = 256) -> bytes:
    """Rows of w (each a multiple of 256 long) as Q4_K blocks, row-major.

    Encoded in chunks of `chunk_blocks` super-blocks so the temporaries stay
    small (large fresh arrays cost more in page faults than in arithmetic)."""
    w = np.ascontiguousarray(w, np.float32)
    assert w.shape[-1] % 256 == 0
    flat = w.reshape(-1, 256)
    return b"".join(_q4k_blocks(flat[i:i + chunk_blocks])
                    for i in range(0, flat.shape[0], chunk_blocks))


def _q4k_blocks(w: np.ndarray) -> bytes:
    x = w.reshape(-1, 8, 32).astype(np.float64)            # [blocks][sub][32]
    lo = np.minimum(x.min(axis=2), 0.0)                     # offsets are subtracted
    hi = x.max(axis=2)
    step = (hi - lo) / 15.0                                 # per sub-block scale
    off = -lo                                               # per sub-block min (>= 0)
    d = step.max(axis=1) / 63.0
    dmin = off.max(axis=1) / 63.0
    d16 = d.astype(np.float16)
    dmin16 = dmin.astype(np.float16)
    d_f = d16.astype(np.float64)
    dmin_f = dmin16.astype(np.float64)
    with np.errstate(divide="ignore", invalid="ignore"):
        sc = np.where(d_f[:, None] > 0, np.rint(step / d_f[:, None]), 0)
        mn = np.where(dmin_f[:, None] > 0, np.rint(off / dmin_f[:, None]), 0)
    sc = np.clip(sc, 0, 63).astype(np.uint8)
    mn = np.clip(mn, 0, 63).astype(np.uint8)
    d1 = d_f[:, None] * sc                                   # effective step
    m1 = dmin_f[:, None] * mn                                # effective offset
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.where(d1[:, :, None] > 0, np.rint((x + m1[:, :, None]) / d1[:, :, None]), 0)
    q = np.clip(q, 0, 15).astype(np.uint8)                  # [blocks][8][32]

    nb = x.shape[0]
    scales = np.zeros((nb, 12), np.uint8)
    scales[:, 0:4] = (sc[:, 0:4] & 63) | ((sc[:, 4:8] >> 4) << 6)
    scales[:, 4:8] = (mn[:, 0:4] & 63) | ((mn[:, 4:8] >> 4) << 6)
    scales[:, 8:12] = (sc[:, 4:8] & 0xF) | ((mn[:, 4:8] & 0xF) << 4)
    qs = (q[:, 0::2, :] | (q[:, 1::2, :] << 4)).reshape(nb, 128)

    blk = np.zeros((nb, 144), np.uint8)
    blk[:, 0:2] = d16.view(np.uint8).reshape(nb, 2)
    blk[:, 2:4] = dmin16.view(np.uint8).reshape(nb, 2)
    blk[:, 4:16] = scales
    blk[:, 16:144] = qs
    return blk.tobytes()


def q4k_decode(data: bytes, n: int) -> np.ndarray:
    """Inverse of q4k_encode (picolm's dequantisation rule), for self-checks."""
    blk = np.frombuffer(data, np.uint8).reshape(-1, 144)
    d = blk[:, 0:2].copy().view(np.float16).astype(np.float32)[:, 0]
    dmin = blk[:, 2:4].copy().view(np.float16).astype(np.float32)[:, 0]
    s = blk[:, 4:16].astype(np.int32)
    sc = np.concatenate([s[:, 0:4] & 63, (s[:, 8:12] & 0xF) | ((s[:, 0:4] >> 6) << 4)], axis=1)
    mn = np.concatenate([s[:, 4:8] & 63, (s[:, 8:12] >> 4) | ((s[:, 4:8] >> 6) << 4)], axis=1)
    qs = blk[:, 16:144].reshape(-1, 4, 32)
    q = np.empty((blk.shape[0], 8, 32), np.float32)
    q[:, 0::2, :] = qs & 0xF
    q[:, 1::2, :] = qs >> 4
    y = (d[:, None] * sc)[:, :, None] * q - (dmin[:, None] * mn)[:, :, None]
    return y.reshape(-1)[:n]


def _str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def write_gguf(path: str, meta: list, tensors: list) -> None:
    """meta: [(key, type, value)]; tensors: [(name, dims, type, nbytes, make)]
    where make() returns the tensor's bytes; tensors are produced one at a
    time while the file is written (only one is held in memory)."""
    head = struct.pack("<IIQQ", GGUF_MAGIC, 3, len(tensors), len(meta))
    for key, t, val in meta:
        head += _str(key) + struct.pack("<I", t)
        if t == T_UINT32:
            head += struct.pack("<I", val)
        elif t == T_FLOAT32:
            head += struct.pack("<f", val)
        elif t == T_STRING:
            head += _str(val)
        else:
            raise ValueError(t)
    off = 0
    for name, dims, t, nbytes, _ in tensors:
        head += _str(name) + struct.pack("<I", len(dims))
        head += b"".join(struct.pack("<Q", d) for d in dims)
        head += struct.pack("<IQ", t, off)
        off += (nbytes + ALIGN - 1) // ALIGN * ALIGN
    with open(path, "wb") as f:
        f.write(head)
        f.write(b"\0" * ((-len(head)) % ALIGN))
        for name, _, _, nbytes, make in tensors:
            data = make()
            if len(data) != nbytes:
                raise ValueError(f"{name}: {len(data)} bytes, header says {nbytes}")
            f.write(data)
            f.write(b"\0" * ((-len(data)) % ALIGN))


def make_model(path: str, layers=22, dim=2048, ffn=5632, heads=32, kv_heads=4, vocab=32000,
               ctx=2048, seed=1, rope_base=10000.0, eps=1e-5) -> None:
    rng = np.random.default_rng(seed)
    hd = dim // heads
    kv_dim = kv_heads * hd

    def q4k(name, rows, cols):  # GGUF dims are (cols, rows): ne0 is the row length
        def make():
            return q4k_encode(rng.standard_normal((rows, cols), dtype=np.float32)
                              * np.float32(0.02))
        return (name, (cols, rows), TYPE_Q4_K, rows * cols // 256 * 144, make)

    def norm(name):
        return (name, (dim,), TYPE_F32, dim * 4, lambda: np.ones(dim, np.float32).tobytes())

    tensors = [q4k("token_embd.weight", vocab, dim)]
    for l in range(layers):
        p = f"blk.{l}."
        tensors += [norm(p + "attn_norm.weight"),
                    q4k(p + "attn_q.weight", dim, dim),
                    q4k(p + "attn_k.weight", kv_dim, dim),
                    q4k(p + "attn_v.weight", kv_dim, dim),
                    q4k(p + "attn_output.weight", dim, dim),
                    norm(p + "ffn_norm.weight"),
                    q4k(p + "ffn_gate.weight", ffn, dim),
                    q4k(p + "ffn_up.weight", ffn, dim),
                    q4k(p + "ffn_down.weight", dim, ffn)]
    tensors += [norm("output_norm.weight"), q4k("output.weight", vocab, dim)]
    meta = [
        ("general.architecture", T_STRING, "llama"),
        ("general.alignment", T_UINT32, ALIGN),
        ("llama.embedding_length", T_UINT32, dim),
        ("llama.feed_forward_length", T_UINT32, ffn),
        ("llama.attention.head_count", T_UINT32, heads),
        ("llama.attention.head_count_kv", T_UINT32, kv_heads),
        ("llama.block_count", T_UINT32, layers),
        ("llama.context_length", T_UINT32, ctx),
        ("llama.rope.freq_base", T_FLOAT32, rope_base),
        ("llama.attention.layer_norm_rms_epsilon", T_FLOAT32, eps),
        ("llama.vocab_size", T_UINT32, vocab),
    ]
    write_gguf(path, meta, tensors)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("out")
    ap.add_argument("--layers", type=int, default=22)
    ap.add_argument("--dim", type=int, default=2048)
    ap.add_argument("--ffn", type=int, default=5632)
    ap.add_argument("--heads", type=int, default=32)
    ap.add_argument("--kv-heads", type=int, default=4)
    ap.add_argument("--vocab", type=int, default=32000)
    ap.add_argument("--ctx", type=int, default=2048)
    ap.add_argument("--seed", type=int, default=1)
    a = ap.parse_args()
    make_model(a.out, a.layers, a.dim, a.ffn, a.heads, a.kv_heads, a.vocab, a.ctx, a.seed)


if __name__ == "__main__":
    main()
