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


# ------------------------------------------------------ projections (GGUF)
GGUF_F32, GGUF_F16, GGUF_Q8_0, GGUF_Q4_K, GGUF_Q6_K = 0, 1, 8, 12, 14
GGUF_TYPES = {"f32": GGUF_F32, "f16": GGUF_F16, "q8_0": GGUF_Q8_0, "q4_k": GGUF_Q4_K,
              "q6_k": GGUF_Q6_K}


def _f16(x) -> np.ndarray:
    return np.asarray(x, np.float32).astype(np.float16).view(np.uint16)


def random_gguf(rng, gtype: int, rows: int, n: int, std: float = 0.02) -> np.ndarray:
    """Raw GGUF rows [rows][row_bytes] (uint8) of type gtype whose
    dequantised weights have roughly standard deviation `std`: random quants
    and block scales in the layouts of picolm/quant.h:65-122."""
    nb = rows * n
    if gtype == GGUF_F32:
        return (rng.standard_normal(nb, dtype=np.float32) * np.float32(std)).view(
            np.uint8).reshape(rows, -1)
    if gtype == GGUF_F16:
        return _f16(rng.standard_normal(nb, dtype=np.float32) * np.float32(std)).view(
            np.uint8).reshape(rows, -1)
    if gtype == GGUF_Q8_0:
        blk = np.empty((nb // 32, 34), np.uint8)
        d = rng.uniform(0.5, 1.5, nb // 32).astype(np.float32) * np.float32(std / 73)
        blk[:, 0:2] = _f16(d).view(np.uint8).reshape(-1, 2)
        blk[:, 2:] = rng.integers(-127, 128, (nb // 32, 32)).astype(np.int8).view(np.uint8)
        return blk.reshape(rows, -1)
    if gtype == GGUF_Q4_K:
        blk = np.empty((nb // 256, 144), np.uint8)
        # weight = d*sc*q - dmin*mn with q, sc, mn uniform: dmin = 7.5 d
        # centres the weights as a quantiser's per-block min does
        d = rng.uniform(0.5, 1.5, nb // 256).astype(np.float32) * np.float32(std / 260)
        dmin = d * np.float32(7.5)
        blk[:, 0:2] = _f16(d).view(np.uint8).reshape(-1, 2)
        blk[:, 2:4] = _f16(dmin).view(np.uint8).reshape(-1, 2)
        blk[:, 4:] = rng.integers(0, 256, (nb // 256, 140), dtype=np.uint8)
        return blk.reshape(rows, -1)
    if gtype == GGUF_Q6_K:
        blk = np.empty((nb // 256, 210), np.uint8)
        blk[:, 0:192] = rng.integers(0, 256, (nb // 256, 192), dtype=np.uint8)
        blk[:, 192:208] = rng.integers(-40, 41, (nb // 256, 16)).astype(np.int8).view(np.uint8)
        d = rng.uniform(0.5, 1.5, nb // 256).astype(np.float32) * np.float32(std / 430)
        blk[:, 208:210] = _f16(d).view(np.uint8).reshape(-1, 2)
        return blk.reshape(rows, -1)
    raise ValueError(gtype)


def random_layer(rng, H, Hk, hd, dim, types=(GGUF_Q4_K,) * 4, bias=False, qk_norm=False,
                 eps=1e-5):
    """One layer's attention weights as the set_layer arguments (dict)."""
    q_dim, kv_dim = H * hd, Hk * hd
    shapes = [(q_dim, dim), (kv_dim, dim), (kv_dim, dim), (dim, q_dim)]
    L = {"dim": dim, "eps": eps, "types": list(types),
         "w": [random_gguf(rng, t, r, n) for t, (r, n) in zip(types, shapes)],
         "attn_norm": (1.0 + 0.1 * rng.standard_normal(dim)).astype(np.float32)}
    for name, rows in (("bq", q_dim), ("bk", kv_dim), ("bv", kv_dim), ("bo", dim)):
        L[name] = (0.1 * rng.standard_normal(rows)).astype(np.float32) if bias else None
    for name in ("q_norm", "k_norm"):
        L[name] = ((1.0 + 0.2 * rng.standard_normal(hd)).astype(np.float32) if qk_norm
                   else None)
    return L


def upload_layer(at, layer, L):
    at.set_layer(layer, L["dim"], L["w"][0], L["types"][0], L["w"][1], L["types"][1],
                 L["w"][2], L["types"][2], L["w"][3], L["types"][3], attn_norm=L["attn_norm"],
                 eps=L["eps"], bq=L["bq"], bk=L["bk"], bv=L["bv"], bo=L["bo"],
                 q_norm=L["q_norm"], k_norm=L["k_norm"])


def oracle_qkv(H, Hk, hd, L, x):
    """model.c:779-817 on one row x: rmsnorm, Q/K/V matmuls + biases, QK-norm."""
    dim, q_dim, kv_dim = L["dim"], H * hd, Hk * hd
    xn = O.rmsnorm(x, L["attn_norm"], L["eps"])
    q = O.matmul(L["w"][0], xn, dim, q_dim, L["types"][0])
    k = O.matmul(L["w"][1], xn, dim, kv_dim, L["types"][1])
    v = O.matmul(L["w"][2], xn, dim, kv_dim, L["types"][2])
    for a, b in ((q, L["bq"]), (k, L["bk"]), (v, L["bv"])):
        if b is not None:
            a += b
    if L["q_norm"] is not None:
        for h in range(H):
            q[h * hd:(h + 1) * hd] = O.rmsnorm(q[h * hd:(h + 1) * hd], L["q_norm"], L["eps"])
        for h in range(Hk):
            k[h * hd:(h + 1) * hd] = O.rmsnorm(k[h * hd:(h + 1) * hd], L["k_norm"], L["eps"])
    return q, k, v


def oracle_out(H, hd, L, x, att):
    """model.c:894-897: x + (Wo att + bo)."""
    y = O.matmul(L["w"][3], att, H * hd, L["dim"], L["types"][3])
    if L["bo"] is not None:
        y += L["bo"]
    return np.asarray(x, np.float32) + y


def assert_kv_near(got, want, what="", max_frac=0.05):
    """KV rows computed from projections that agree with picolm's to FP32
    rounding.  Each FP16 value may differ from the oracle's by one FP16 unit
    (the FP32 value at a rounding boundary) plus 4e-6 of the row's RMS (the
    FP32 rounding of the projection itself, which is several FP16 units for
    values near zero).  Over the rows passed together, at most max_frac of
    the words may differ at all (about 1.5% do on the tensor-core path,
    whose in-MMA accumulation rounds a little coarser than sequential FP32;
    pass many rows at once for a meaningful fraction)."""
    got = np.asarray(got, np.uint16)
    want = np.asarray(want, np.uint16)
    g = O.fp16_to_fp32(got).reshape(got.shape).astype(np.float64)
    w = O.fp16_to_fp32(want).reshape(want.shape).astype(np.float64)
    rms = np.sqrt(np.mean(w * w, axis=-1, keepdims=True))
    ulp = np.spacing(np.abs(w).astype(np.float16)).astype(np.float64)
    err = np.abs(g - w)
    bad = err > ulp + 4e-6 * rms
    assert not bad.any(), (f"{what}: {int(bad.sum())} FP16 values off by more than one unit "
                           f"+ 4e-6 rms (worst {err[bad].max():.3e} at {w[bad][0]:.3e})")
    frac = float((got != want).mean())
    assert frac <= max_frac, f"{what}: {frac:.2%} of FP16 words differ"
