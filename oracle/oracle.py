"""ctypes bindings for the CPU oracle -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module, and only as the checker.  The product (picolm_b200 and
libpl_attn.so) never loads it.

Two libraries:
  * ``libpl_oracle.so``   -- the C restatement of picolm's attention path
    (oracle/pl_oracle.c), built by ``make -C oracle``;
  * ``_ref/libpicoref.so`` -- the genuine picolm sources compiled in place
    from the reference tree (``make -C oracle ref``).  It exists only where
    the reference tree was present at build time.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PORT_SO = os.path.join(HERE, "libpl_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libpicoref.so")

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")


class OrcCfg(C.Structure):
    _fields_ = [("n_heads", C.c_int), ("n_kv_heads", C.c_int),
                ("head_dim", C.c_int), ("max_seq", C.c_int),
                ("rope_type", C.c_int)]


def build_port() -> None:
    subprocess.run(["make", "-s", "-C", HERE, "all"], check=True)


_port = None
_ref = None


def port() -> C.CDLL:
    """The C restatement (oracle/pl_oracle.c)."""
    global _port
    if _port is None:
        if not os.path.exists(PORT_SO):
            build_port()
        lib = C.CDLL(PORT_SO)
        lib.orc_fp16_to_fp32.restype = C.c_float
        lib.orc_fp16_to_fp32.argtypes = [C.c_uint16]
        lib.orc_fp32_to_fp16.restype = C.c_uint16
        lib.orc_fp32_to_fp16.argtypes = [C.c_float]
        lib.orc_fp32_to_fp16_array.argtypes = [_f32p, _u16p, C.c_long]
        lib.orc_fp16_to_fp32_array.argtypes = [_u16p, _f32p, C.c_long]
        lib.orc_rope_tables.argtypes = [_f32p, _f32p, C.c_int, C.c_int, C.c_float]
        lib.orc_rope.argtypes = [_f32p, _f32p, C.c_int, C.c_int, C.c_int,
                                 _f32p, _f32p, C.c_int]
        cfgp = C.POINTER(OrcCfg)
        lib.orc_attn_decode.argtypes = [cfgp, _u16p, _u16p, C.c_int, _f32p, _f32p,
                                        _f32p, _f32p, _f32p, _f32p]
        lib.orc_attn_core.argtypes = [cfgp, _u16p, _u16p, C.c_int, _f32p, _f32p]
        lib.orc_attn_prefill.argtypes = [cfgp, _u16p, _u16p, C.c_int, C.c_int,
                                         _f32p, _f32p, _f32p, _f32p, _f32p, _f32p,
                                         C.c_int]
        lib.orc_attn_decode_seqs.argtypes = [cfgp, C.c_int, _u16p, _u16p, C.c_long,
                                             _i32p, _f32p, _f32p, _f32p, _f32p,
                                             _f32p, _f32p, C.c_int]
        lib.orc_matvec.argtypes = [_f32p, _f32p, _f32p, C.c_int, C.c_int]
        lib.orc_vec_dot.restype = C.c_float
        lib.orc_vec_dot.argtypes = [C.c_void_p, _f32p, C.c_int, C.c_int]
        lib.orc_row_bytes.restype = C.c_long
        lib.orc_row_bytes.argtypes = [C.c_int, C.c_int]
        lib.orc_matmul.argtypes = [_f32p, _f32p, C.c_void_p, C.c_int, C.c_int, C.c_int]
        lib.orc_rmsnorm.argtypes = [_f32p, _f32p, _f32p, C.c_int, C.c_float]
        _port = lib
    return _port


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def ref() -> C.CDLL:
    """The genuine picolm code compiled from the reference tree."""
    global _ref
    if _ref is None:
        lib = C.CDLL(REF_SO)
        lib.fp32_to_fp16.restype = C.c_uint16
        lib.fp32_to_fp16.argtypes = [C.c_float]
        lib.fp16_to_fp32.restype = C.c_float
        lib.fp16_to_fp32.argtypes = [C.c_uint16]
        lib.rope.argtypes = [_f32p, _f32p, C.c_int, C.c_int, C.c_int, _f32p, _f32p,
                             C.c_int]
        lib.ref_fp32_to_fp16_array.argtypes = [_f32p, _u16p, C.c_long]
        lib.ref_fp16_to_fp32_array.argtypes = [_u16p, _f32p, C.c_long]
        lib.ref_rope_tables.argtypes = [_f32p, _f32p, C.c_int, C.c_int, C.c_float]
        lib.ref_decode_layer.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.c_float,
                                         C.c_int, _f32p, _f32p, _f32p, _f32p, _u16p,
                                         _u16p, C.c_int, _f32p, _f32p, _f32p, _f32p,
                                         _f32p, _f32p]
        lib.ref_prefill_layer.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int,
                                          C.c_float, C.c_int, _f32p, C.c_int, C.c_int,
                                          _f32p, _f32p, _f32p, _u16p, _u16p, _f32p,
                                          _f32p, _f32p]
        lib.ref_attn_decode_seqs.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, _u16p,
                                             _u16p, C.c_long, _i32p, _f32p, _f32p,
                                             _f32p, _f32p, _f32p, _f32p, C.c_int]
        lib.ref_attn_prefill_seqs.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, _u16p,
                                              _u16p, C.c_long, C.c_int, C.c_int, _f32p,
                                              _f32p, _f32p, _f32p, _f32p, _f32p, C.c_int]
        lib.matmul.argtypes = [_f32p, _f32p, C.c_void_p, C.c_int, C.c_int, C.c_int]
        lib.vec_dot.restype = C.c_float
        lib.vec_dot.argtypes = [C.c_void_p, _f32p, C.c_int, C.c_int]
        lib.rmsnorm.argtypes = [_f32p, _f32p, _f32p, C.c_int, C.c_float]
        _ref = lib
    return _ref


# ---------------------------------------------------------------- helpers
def cfg(n_heads, n_kv_heads, head_dim, max_seq, rope_type=0) -> OrcCfg:
    return OrcCfg(n_heads, n_kv_heads, head_dim, max_seq, rope_type)


def ctypes_ref(c: OrcCfg):
    """A config as the pointer argument of the orc_* functions."""
    return C.byref(c)


def fp32_to_fp16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    out = np.empty(x.size, np.uint16)
    port().orc_fp32_to_fp16_array(x, out, x.size)
    return out


def fp16_to_fp32(h: np.ndarray) -> np.ndarray:
    h = np.ascontiguousarray(h, dtype=np.uint16).ravel()
    out = np.empty(h.size, np.float32)
    port().orc_fp16_to_fp32_array(h, out, h.size)
    return out


def rope_tables(max_seq: int, head_dim: int, base: float):
    half = head_dim // 2
    c = np.empty(max_seq * half, np.float32)
    s = np.empty(max_seq * half, np.float32)
    port().orc_rope_tables(c, s, max_seq, head_dim, base)
    return c, s


def attn_decode(c: OrcCfg, kc, vc, pos, q, k, v, cos_t, sin_t):
    """Returns (out, q_rot, k_rot); kc/vc (layer views) are updated in place."""
    q = np.array(q, np.float32).ravel()
    k = np.array(k, np.float32).ravel()
    v = np.ascontiguousarray(v, np.float32).ravel()
    out = np.empty(c.n_heads * c.head_dim, np.float32)
    port().orc_attn_decode(C.byref(c), kc, vc, int(pos), q, k, v, cos_t, sin_t, out)
    return out, q, k


def attn_prefill(c: OrcCfg, kc, vc, start_pos, q, k, v, cos_t, sin_t):
    """q [n][H*hd], k/v [n][kv_dim]; returns (out [n][H*hd], q_rot, k_rot)."""
    q = np.array(q, np.float32)
    k = np.array(k, np.float32)
    v = np.ascontiguousarray(v, np.float32)
    n = q.shape[0]
    qd = c.n_heads * c.head_dim
    out = np.empty((n, qd), np.float32)
    port().orc_attn_prefill(C.byref(c), kc, vc, int(start_pos), n, q.ravel(), k.ravel(),
                            v.ravel(), cos_t, sin_t, out.ravel(), qd)
    return out, q, k


def attn_decode_seqs(c: OrcCfg, kc, vc, seq_stride, pos, q, k, v, cos_t, sin_t,
                     n_threads=1, use_ref=False):
    """Batched decode over independent sequences; kc/vc flat uint16."""
    n_seq = len(pos)
    pos = np.ascontiguousarray(pos, np.int32)
    q = np.array(q, np.float32).ravel()
    k = np.array(k, np.float32).ravel()
    v = np.ascontiguousarray(v, np.float32).ravel()
    out = np.empty(n_seq * c.n_heads * c.head_dim, np.float32)
    if use_ref:
        ref().ref_attn_decode_seqs(c.n_heads, c.n_kv_heads, c.head_dim, n_seq, kc, vc,
                                   int(seq_stride), pos, q, k, v, cos_t, sin_t, out,
                                   int(n_threads))
    else:
        port().orc_attn_decode_seqs(C.byref(c), n_seq, kc, vc, int(seq_stride), pos, q,
                                    k, v, cos_t, sin_t, out, int(n_threads))
    return out


def attn_prefill_seqs(c: OrcCfg, kc, vc, seq_stride, start_pos, n_tok, q, k, v, cos_t, sin_t,
                      n_threads=1, use_ref=False):
    """Causal prefill of n_seq independent sequences (flat uint16 caches,
    slab s at s*seq_stride; q [n_seq][n_tok][H*hd], k/v [n_seq][n_tok][kv_dim])
    over n_threads threads, one sequence per thread at a time."""
    q = np.array(q, np.float32)
    k = np.array(k, np.float32)
    v = np.ascontiguousarray(v, np.float32)
    n_seq = q.shape[0]
    qd = c.n_heads * c.head_dim
    out = np.empty((n_seq, n_tok, qd), np.float32)
    if use_ref:
        ref().ref_attn_prefill_seqs(c.n_heads, c.n_kv_heads, c.head_dim, n_seq, kc, vc,
                                    int(seq_stride), int(start_pos), int(n_tok), q.ravel(),
                                    k.ravel(), v.ravel(), cos_t, sin_t, out.ravel(),
                                    int(n_threads))
        return out
    from concurrent.futures import ThreadPoolExecutor
    kv_dim = c.n_kv_heads * c.head_dim

    def one(s):
        sl = slice(s * seq_stride, (s + 1) * seq_stride)
        o = np.empty((n_tok, qd), np.float32)
        port().orc_attn_prefill(C.byref(c), kc[sl], vc[sl], int(start_pos), int(n_tok),
                                q[s].ravel(), k[s].ravel(), v[s].reshape(-1, kv_dim).ravel(),
                                cos_t, sin_t, o.ravel(), qd)
        out[s] = o

    with ThreadPoolExecutor(max(1, int(n_threads))) as ex:
        list(ex.map(one, range(n_seq)))
    return out


# ------------------------------------------------- projections (GGUF GEMV)
def matmul(W: np.ndarray, x, n: int, d: int, gtype: int, use_ref: bool = False) -> np.ndarray:
    """out[d] = W x for raw GGUF rows W (bytes) of type gtype, as picolm's
    matmul; the restatement, or the genuine reference with use_ref."""
    W = np.ascontiguousarray(W)
    x = np.ascontiguousarray(x, np.float32).ravel()
    out = np.empty(d, np.float32)
    if use_ref:
        ref().matmul(out, x, W.ctypes.data, n, d, gtype)
    else:
        port().orc_matmul(out, x, W.ctypes.data, n, d, gtype)
    return out


def rmsnorm(x, w, eps: float, use_ref: bool = False) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32).ravel()
    w = np.ascontiguousarray(w, np.float32).ravel()
    out = np.empty_like(x)
    (ref().rmsnorm if use_ref else port().orc_rmsnorm)(out, x, w, x.size, float(eps))
    return out


def row_bytes(gtype: int, n: int) -> int:
    return int(port().orc_row_bytes(gtype, n))
