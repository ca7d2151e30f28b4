"""Helpers shared by the GPU parity tests."""
import numpy as np

from oracle import oracle as O

# Tolerance from the north-star spec: attention output within max-abs 2e-3
# and rel 1e-2 (FP32 accumulation).  Checked element-wise as
# |got - want| <= ATOL + RTOL*|want| AND max |got - want| <= ATOL.
ATOL = 2e-3
RTOL = 1e-2


def assert_attn_close(got, want, what=""):
    got = np.asarray(got, np.float32)
    want = np.asarray(want, np.float32)
    assert got.shape == want.shape, (got.shape, want.shape)
    assert np.all(np.isfinite(got)), f"{what}: non-finite output"
    err = np.abs(got.astype(np.float64) - want.astype(np.float64))
    max_abs = float(err.max()) if err.size else 0.0
    assert max_abs <= ATOL, f"{what}: max abs err {max_abs:.3e} > {ATOL}"
    assert np.all(err <= ATOL + RTOL * np.abs(want)), f"{what}: rel check failed"
    return max_abs


def random_cache(rng, n_rows, kv_dim, scale=1.0):
    """FP16 (picolm rounding) cache rows [n_rows][kv_dim], ~N(0, scale)."""
    x = rng.standard_normal((n_rows, kv_dim), dtype=np.float32) * np.float32(scale)
    return O.fp32_to_fp16(x).reshape(n_rows, kv_dim)


def oracle_decode_layer(H, Hk, ms, kc, vc, pos, q, k, v, tables, rope_type=0, hd=64):
    """Oracle decode on copies of the layer views; returns (out, kc', vc')."""
    c = O.cfg(H, Hk, hd, ms, rope_type)
    kc2, vc2 = kc.copy(), vc.copy()
    out, _, _ = O.attn_decode(c, kc2.ravel(), vc2.ravel(), pos, q, k, v, *tables)
    return out, kc2, vc2
