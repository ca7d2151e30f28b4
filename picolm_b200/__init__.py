"""picolm_b200 -- B200 attention hot path for picolm, behind a C ABI.

The product is the shared library ``libpl_attn.so`` built from
``picolm_b200/csrc`` (see ``include/pl_attn.h`` for the C interface).  This
module is a thin ctypes binding over that C ABI for Python callers, the test
suite and the benchmark: every call goes straight into the CUDA library.
There is no CPU path: if the library is missing, cannot be loaded, or has
no usable sm_100 device, calls raise :class:`PlAttnError`.

``Attn`` mirrors the C entry points one for one and keeps their argument
meaning; host-buffer methods take numpy arrays, ``*_dev`` methods take raw
device pointers (ints), e.g. ``torch.Tensor.data_ptr()``.
"""
from __future__ import annotations

import ctypes as C
import os
import re

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libpl_attn.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "pl_attn.h")

PL_OK = 0
PL_EFAIL = -1
PL_EARG = -2
PL_ENOMEM = -3
PL_ECUDA = -4
PL_ETIMEOUT = -5
PL_ESTATE = -6
PL_EDEVICE = -7
PL_EUNSUPPORTED = -8
PL_ROPE_LLAMA = 0
PL_ROPE_QWEN = 1
PL_SPLIT_SEQS = 0
PL_SPLIT_KV = 1
# GGUF tensor types the projections take (picolm/quant.h:49-63)
PL_GGUF_F32 = 0
PL_GGUF_F16 = 1
PL_GGUF_Q8_0 = 8
PL_GGUF_Q4_K = 12
PL_GGUF_Q6_K = 14
HEAD_DIM = 64                # default head_dim; 64 and 128 are supported
PART_STRIDE = HEAD_DIM + 4   # floats per partial at head_dim 64: m, l, 2 pad, o[64]


def part_stride(head_dim: int = HEAD_DIM) -> int:
    """Floats per head in a partial block: m, l, 2 pad, o[head_dim]."""
    return head_dim + 4


class PlAttnError(RuntimeError):
    def __init__(self, rc: int, what: str):
        self.rc = rc
        super().__init__(f"{what}: {strerror(rc)} ({rc})")


_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_vp = C.c_void_p
_lib = None


def declared_symbols() -> list[str]:
    """Names of the functions include/pl_attn.h declares (non-stub part)."""
    text = open(HEADER).read()
    text = text.split("#else /* PL_ATTN_DISABLED")[0]
    return sorted(set(re.findall(r"\b(pl_[a-z0-9_]+)\s*\(", text)))


def load(path: str = LIB_PATH) -> C.CDLL:
    """Load libpl_attn.so and declare its signatures.  Raises if absent."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise PlAttnError(PL_EDEVICE, f"{path} is missing; run python -m picolm_b200.build")
    lib = C.CDLL(path)
    i = C.c_int
    sig = {
        "pl_attn_host_register": (i, [C.c_void_p, C.c_size_t]),
        "pl_attn_host_unregister": (i, [C.c_void_p]),
        "pl_attn_init": (i, [i, i, i, i, i, C.c_float, i, i, i]),
        "pl_attn_init_devices": (i, [i, i, i, i, i, C.c_float, i, i, i, _i32p, i]),
        "pl_attn_set_rope": (i, [_f32p, _f32p, i, i]),
        "pl_attn_available": (i, []),
        "pl_attn_shutdown": (None, []),
        "pl_attn_strerror": (C.c_char_p, [i]),
        "pl_attn_decode": (i, [i, i, i, _f32p, _f32p, _f32p, _f32p]),
        "pl_attn_decode_batch": (i, [i, i, _i32p, _i32p, _f32p, _f32p, _f32p, _f32p]),
        "pl_attn_prefill": (i, [i, i, i, i, _f32p, _f32p, _f32p, _f32p, i]),
        "pl_attn_rope": (i, [i, i, _vp, _vp]),
        "pl_kv_download": (i, [i, i, i, i, _vp, _vp]),
        "pl_kv_upload": (i, [i, i, i, i, _vp, _vp]),
        "pl_attn_decode_batch_dev": (i, [i, i, _vp, _vp, i, _vp, _vp, _vp, _vp, _vp]),
        "pl_attn_prefill_dev": (i, [i, i, i, i, _vp, _vp, _vp, _vp, i, _vp]),
        "pl_attn_decode_partial_dev": (i, [i, i, i, i, i, i, _vp, _vp, _vp, _vp, _vp]),
        "pl_attn_combine_dev": (i, [i, _vp, _vp, _vp]),
        "pl_attn_kv_ptr": (i, [i, i, C.POINTER(_vp), C.POINTER(_vp)]),
        "pl_attn_xfer_handle_bytes": (i, []),
        "pl_attn_xfer_setup": (i, [i, i, _vp]),
        "pl_attn_xfer_connect": (i, [_vp]),
        "pl_attn_combine_p2p_dev": (i, [_vp, _vp, _vp]),
        "pl_attn_decode_p2p_dev": (i, [i, i, i, i, i, i, _vp, _vp, _vp, _vp, _vp]),
        "pl_attn_decode_batch_dev_noalloc": (i, [i, i, _vp, _vp, i, _vp, _vp, _vp, _vp, _vp]),
        "pl_attn_set_layer": (i, [i, i, _vp, C.c_float, _vp, i, _vp, i, _vp, i, _vp, i,
                                  _vp, _vp, _vp, _vp, _vp, _vp]),
        "pl_attn_block_decode": (i, [i, i, _i32p, _i32p, _f32p]),
        "pl_attn_block_prefill": (i, [i, i, i, i, _f32p]),
        "pl_attn_block_decode_dev": (i, [i, i, _vp, _vp, i, _vp, _vp]),
        "pl_attn_block_prefill_dev": (i, [i, i, i, i, _vp, _vp]),
        "pl_attn_proj": (i, [i, i, i, _f32p, _f32p]),
        "pl_attn_status": (i, [_vp]),
        "pl_attn_set_wait_limit": (i, [C.c_double]),
        "pl_attn_profile": (i, [i]),
        "pl_attn_profile_read": (i, [C.POINTER(C.c_double), C.POINTER(C.c_long),
                                     C.POINTER(C.c_long)]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def strerror(rc: int) -> str:
    try:
        return load().pl_attn_strerror(rc).decode()
    except Exception:  # library itself unavailable
        return f"status {rc}"


def _check(rc: int, what: str) -> None:
    if rc != PL_OK:
        raise PlAttnError(rc, what)


def _ptr(a) -> int | None:
    """numpy array -> host address (None passes NULL)."""
    if a is None:
        return None
    return a.ctypes.data


class Attn:
    """The module context (one per process, like picolm's gpu.c state)."""

    def __init__(self, n_layers: int, n_heads: int, n_kv_heads: int, max_seq: int,
                 rope_base: float = 10000.0, rope_type: int = PL_ROPE_LLAMA,
                 n_seqs: int = 1, device: int = 0, head_dim: int = HEAD_DIM,
                 devices=None, split: int = PL_SPLIT_SEQS):
        """pl_attn_init on `device`, or pl_attn_init_devices over the list
        `devices` (ids may repeat) with `split` PL_SPLIT_SEQS / PL_SPLIT_KV."""
        self.lib = load()
        self.n_layers, self.n_heads, self.n_kv_heads = n_layers, n_heads, n_kv_heads
        self.head_dim, self.max_seq, self.n_seqs = head_dim, max_seq, n_seqs
        self.q_dim = n_heads * head_dim
        self.kv_dim = n_kv_heads * head_dim
        self.part_stride = part_stride(head_dim)
        if devices is None:
            _check(self.lib.pl_attn_init(n_layers, n_heads, n_kv_heads, head_dim, max_seq,
                                         float(rope_base), rope_type, n_seqs, device),
                   "pl_attn_init")
        else:
            devs = np.ascontiguousarray(devices, np.int32)
            _check(self.lib.pl_attn_init_devices(n_layers, n_heads, n_kv_heads, head_dim,
                                                 max_seq, float(rope_base), rope_type, n_seqs,
                                                 devs.size, devs, split),
                   "pl_attn_init_devices")
        self._open = True

    # lifecycle ---------------------------------------------------------
    def close(self) -> None:
        if self._open:
            self.lib.pl_attn_shutdown()
            self._open = False

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def set_rope(self, cos_tab: np.ndarray, sin_tab: np.ndarray) -> None:
        half = self.head_dim // 2
        c = np.ascontiguousarray(cos_tab, np.float32).ravel()
        s = np.ascontiguousarray(sin_tab, np.float32).ravel()
        _check(self.lib.pl_attn_set_rope(c, s, c.size // half, half), "pl_attn_set_rope")

    # host-buffer entry points -----------------------------------------
    def decode(self, seq: int, layer: int, pos: int, q, k, v) -> np.ndarray:
        out = np.empty(self.q_dim, np.float32)
        _check(self.lib.pl_attn_decode(seq, layer, pos, _f32(q), _f32(k), _f32(v), out),
               "pl_attn_decode")
        return out

    def decode_batch(self, layer: int, seqs, pos, q, k, v, out=None) -> np.ndarray:
        """`out` (float32, n*q_dim, contiguous) is reused if given, as a
        caller such as model.c reuses its s->xb."""
        seqs = np.ascontiguousarray(seqs, np.int32)
        pos = np.ascontiguousarray(pos, np.int32)
        n = seqs.size
        if out is None:
            out = np.empty(n * self.q_dim, np.float32)
        elif out.dtype != np.float32 or not out.flags.c_contiguous or out.size != n * self.q_dim:
            raise ValueError("out must be a contiguous float32 array of n * q_dim")
        _check(self.lib.pl_attn_decode_batch(layer, n, seqs, pos, _f32(q), _f32(k), _f32(v),
                                             out), "pl_attn_decode_batch")
        return out.reshape(n, self.q_dim)

    def prefill(self, seq: int, layer: int, start_pos: int, q, k, v,
                out_stride: int | None = None, out=None) -> np.ndarray:
        """`out` (float32, n_tok*out_stride, contiguous) is reused if given."""
        q = _f32(q)
        n_tok = q.size // self.q_dim
        stride = self.q_dim if out_stride is None else out_stride
        if out is None:
            out = np.zeros(n_tok * stride, np.float32)
        elif out.dtype != np.float32 or not out.flags.c_contiguous or out.size != n_tok * stride:
            raise ValueError("out must be a contiguous float32 array of n_tok * out_stride")
        _check(self.lib.pl_attn_prefill(seq, layer, start_pos, n_tok, q, _f32(k), _f32(v),
                                        out, stride), "pl_attn_prefill")
        return out.reshape(n_tok, stride)

    def rope(self, pos0: int, q=None, k=None):
        qa = None if q is None else np.array(q, np.float32)
        ka = None if k is None else np.array(k, np.float32)
        n_tok = (qa.size // self.q_dim) if qa is not None else (ka.size // self.kv_dim)
        _check(self.lib.pl_attn_rope(pos0, n_tok, _ptr(qa), _ptr(ka)), "pl_attn_rope")
        return qa, ka

    def host_register(self, arr: np.ndarray) -> None:
        """Page-lock `arr` (a contiguous array the caller keeps alive) so
        that host-buffer calls move it without staging."""
        if not arr.flags.c_contiguous:
            raise ValueError("host_register needs a contiguous array")
        _check(self.lib.pl_attn_host_register(arr.ctypes.data, arr.nbytes),
               "pl_attn_host_register")

    def host_unregister(self, arr: np.ndarray) -> None:
        _check(self.lib.pl_attn_host_unregister(arr.ctypes.data), "pl_attn_host_unregister")

    def kv_download(self, seq: int, layer: int, pos0: int, n_pos: int):
        k = np.empty(n_pos * self.kv_dim, np.uint16)
        v = np.empty(n_pos * self.kv_dim, np.uint16)
        _check(self.lib.pl_kv_download(seq, layer, pos0, n_pos, _ptr(k), _ptr(v)),
               "pl_kv_download")
        return k.reshape(n_pos, self.kv_dim), v.reshape(n_pos, self.kv_dim)

    def kv_upload(self, seq: int, layer: int, pos0: int, k, v) -> None:
        k = np.ascontiguousarray(k, np.uint16)
        v = np.ascontiguousarray(v, np.uint16)
        n_pos = k.size // self.kv_dim
        _check(self.lib.pl_kv_upload(seq, layer, pos0, n_pos, _ptr(k), _ptr(v)),
               "pl_kv_upload")

    # the attention sub-block with its projections ----------------------
    def set_layer(self, layer: int, dim: int, wq, type_q: int, wk, type_k: int, wv,
                  type_v: int, wo, type_o: int, attn_norm=None, eps: float = 1e-5,
                  bq=None, bk=None, bv=None, bo=None, q_norm=None, k_norm=None) -> None:
        """Upload one layer's attention weights: w* are raw GGUF row bytes
        (numpy arrays of any dtype, contiguous) of GGUF type type_*; norms
        and biases float32 or None."""
        ws = [np.ascontiguousarray(w) for w in (wq, wk, wv, wo)]
        fs = [None if a is None else _f32(a) for a in (attn_norm, bq, bk, bv, bo, q_norm, k_norm)]
        p = [None if a is None else a.ctypes.data for a in fs]
        _check(self.lib.pl_attn_set_layer(layer, dim, p[0], float(eps),
                                          ws[0].ctypes.data, type_q, ws[1].ctypes.data, type_k,
                                          ws[2].ctypes.data, type_v, ws[3].ctypes.data, type_o,
                                          p[1], p[2], p[3], p[4], p[5], p[6]),
               "pl_attn_set_layer")

    def block_decode(self, layer: int, seqs, pos, x) -> np.ndarray:
        """x [n][dim] residual stream; returns x + attention sub-block(x)
        (a new array; the argument is not modified)."""
        seqs = np.ascontiguousarray(seqs, np.int32)
        pos = np.ascontiguousarray(pos, np.int32)
        xo = np.array(x, np.float32, order="C")
        _check(self.lib.pl_attn_block_decode(layer, seqs.size, seqs, pos, xo.ravel()),
               "pl_attn_block_decode")
        return xo.reshape(seqs.size, -1)

    def block_prefill(self, seq: int, layer: int, start_pos: int, x) -> np.ndarray:
        xo = np.array(x, np.float32, order="C")
        n_tok = xo.shape[0] if xo.ndim == 2 else 1
        _check(self.lib.pl_attn_block_prefill(seq, layer, start_pos, n_tok, xo.ravel()),
               "pl_attn_block_prefill")
        return xo.reshape(n_tok, -1)

    def block_decode_dev(self, layer, n, d_seqs, d_pos, max_pos, d_x, stream=None) -> None:
        _check(self.lib.pl_attn_block_decode_dev(layer, n, d_seqs, d_pos, max_pos, d_x, stream),
               "pl_attn_block_decode_dev")

    def block_prefill_dev(self, seq, layer, start_pos, n_tok, d_x, stream=None) -> None:
        _check(self.lib.pl_attn_block_prefill_dev(seq, layer, start_pos, n_tok, d_x, stream),
               "pl_attn_block_prefill_dev")

    def proj(self, layer: int, which: int, x, rows: int) -> np.ndarray:
        """matmul_bias with uploaded weight `which` (0 q, 1 k, 2 v, 3 o) on
        the rows of x; rows = output rows of that weight."""
        xa = np.array(x, np.float32, order="C")
        n = xa.shape[0] if xa.ndim == 2 else 1
        y = np.empty(n * rows, np.float32)
        _check(self.lib.pl_attn_proj(layer, which, n, xa.ravel(), y), "pl_attn_proj")
        return y.reshape(n, rows)

    def raw(self):
        """The C entry points with plain void* arguments (a second ctypes view
        of the same library, without numpy argument conversion): what a thin
        FFI binding of the C ABI costs per call, e.g. raw().pl_attn_decode_batch(
        layer, n, seqs_ptr, pos_ptr, q_ptr, k_ptr, v_ptr, out_ptr)."""
        if getattr(self, "_raw", None) is None:
            lib = C.CDLL(LIB_PATH)
            lib.pl_attn_decode_batch.restype = C.c_int
            lib.pl_attn_decode_batch.argtypes = [C.c_int, C.c_int] + [C.c_void_p] * 6
            lib.pl_attn_decode.restype = C.c_int
            lib.pl_attn_decode.argtypes = [C.c_int, C.c_int, C.c_int] + [C.c_void_p] * 4
            lib.pl_attn_prefill.restype = C.c_int
            lib.pl_attn_prefill.argtypes = [C.c_int] * 4 + [C.c_void_p] * 4 + [C.c_int]
            self._raw = lib
        return self._raw

    # status and failure detection -------------------------------------
    def status(self, stream=None) -> int:
        """pl_attn_status: wait for `stream`, read and clear the device
        error word; returns the status code (PL_OK, PL_ETIMEOUT, PL_EARG)."""
        return self.lib.pl_attn_status(stream)

    def set_wait_limit(self, seconds: float) -> None:
        _check(self.lib.pl_attn_set_wait_limit(float(seconds)), "pl_attn_set_wait_limit")

    # device-pointer entry points --------------------------------------
    def decode_batch_dev(self, layer, n, d_seqs, d_pos, max_pos, d_q, d_k, d_v, d_out,
                         stream=None) -> None:
        _check(self.lib.pl_attn_decode_batch_dev(layer, n, d_seqs, d_pos, max_pos, d_q, d_k,
                                                 d_v, d_out, stream),
               "pl_attn_decode_batch_dev")

    def decode_batch_dev_noalloc(self, layer, n, d_seqs, d_pos, max_pos, d_q, d_k, d_v,
                                 d_out, stream=None) -> None:
        """decode_batch_dev without any device allocation (fixed static scratch:
        n <= 1024, split partials capped at 4 MiB; calls sharing it must not
        overlap on the GPU)."""
        _check(self.lib.pl_attn_decode_batch_dev_noalloc(layer, n, d_seqs, d_pos, max_pos, d_q,
                                                         d_k, d_v, d_out, stream),
               "pl_attn_decode_batch_dev_noalloc")

    def prefill_dev(self, seq, layer, start_pos, n_tok, d_q, d_k, d_v, d_out,
                    out_stride=None, stream=None) -> None:
        stride = self.q_dim if out_stride is None else out_stride
        _check(self.lib.pl_attn_prefill_dev(seq, layer, start_pos, n_tok, d_q, d_k, d_v, d_out,
                                            stride, stream), "pl_attn_prefill_dev")

    def decode_partial_dev(self, seq, layer, pos, row0, n_rows, append, d_q, d_k, d_v,
                           d_part, stream=None) -> None:
        _check(self.lib.pl_attn_decode_partial_dev(seq, layer, pos, row0, n_rows,
                                                   1 if append else 0, d_q, d_k, d_v, d_part,
                                                   stream), "pl_attn_decode_partial_dev")

    def combine_dev(self, n_part, d_parts, d_out, stream=None) -> None:
        _check(self.lib.pl_attn_combine_dev(n_part, d_parts, d_out, stream),
               "pl_attn_combine_dev")

    def profile(self, enable: bool = True) -> None:
        _check(self.lib.pl_attn_profile(1 if enable else 0), "pl_attn_profile")

    def profile_read(self):
        """(attention-kernel ms, attention launches, all launches) since last read."""
        ms, na, nl = C.c_double(), C.c_long(), C.c_long()
        _check(self.lib.pl_attn_profile_read(C.byref(ms), C.byref(na), C.byref(nl)),
               "pl_attn_profile_read")
        return ms.value, na.value, nl.value

    def xfer_setup(self, world: int, rank: int) -> bytes:
        """Receive buffer of the P2P KV-split merge; returns its IPC handle."""
        buf = C.create_string_buffer(self.lib.pl_attn_xfer_handle_bytes())
        _check(self.lib.pl_attn_xfer_setup(world, rank, buf), "pl_attn_xfer_setup")
        return buf.raw

    def xfer_connect(self, handles) -> None:
        """Map the other ranks' buffers; `handles` in rank order."""
        blob = C.create_string_buffer(b"".join(handles))
        _check(self.lib.pl_attn_xfer_connect(blob), "pl_attn_xfer_connect")

    def combine_p2p_dev(self, d_part, d_out, stream=None) -> None:
        _check(self.lib.pl_attn_combine_p2p_dev(d_part, d_out, stream),
               "pl_attn_combine_p2p_dev")

    def decode_p2p_dev(self, seq, layer, pos, row0, n_rows, append, d_q, d_k, d_v, d_out,
                       stream=None) -> None:
        _check(self.lib.pl_attn_decode_p2p_dev(seq, layer, pos, row0, n_rows, int(append), d_q,
                                               d_k, d_v, d_out, stream),
               "pl_attn_decode_p2p_dev")

    def kv_ptr(self, seq: int, layer: int):
        k = _vp()
        v = _vp()
        _check(self.lib.pl_attn_kv_ptr(seq, layer, C.byref(k), C.byref(v)), "pl_attn_kv_ptr")
        return k.value, v.value


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, np.float32).ravel()
