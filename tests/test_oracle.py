"""The CPU oracle against the genuine picolm reference (CPU only).

Pins oracle/pl_oracle.c against tests/golden/golden.npz, which
tests/golden/make_golden.py produced from picolm's own quant.c / tensor.c /
model.c.  Every comparison is bit-exact.  When oracle/_ref (the reference
compiled here) is present, the oracle is also checked live against it on
fresh random inputs.
"""
import hashlib

import numpy as np
import pytest

from tests.golden.make_golden import f16_encode_patterns


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def test_fp16_encode_special_values(golden, orc):
    # quant.c:41-78: ties away from zero, subnormal handling, NaN/Inf/overflow
    got = orc.fp32_to_fp16(golden["f16_special_in"])
    np.testing.assert_array_equal(got, golden["f16_special_out"])


def test_fp16_encode_ties_away_from_zero(orc):
    # 1 + 2^-11 is an exact FP16 tie; RNE gives 0x3C00, picolm gives 0x3C01
    assert orc.port().orc_fp32_to_fp16(1.0 + 2.0 ** -11) == 0x3C01
    assert orc.port().orc_fp32_to_fp16(-(1.0 + 2.0 ** -11)) == 0xBC01


def test_fp16_encode_patterns_digest(golden, orc):
    pats = f16_encode_patterns()
    assert pats.size == int(golden["f16_enc_patterns_n"])
    assert sha(orc.fp32_to_fp16(pats)) == str(golden["f16_enc_patterns_sha"])


def test_fp16_decode_all_halves_digest(golden, orc):
    h = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    assert sha(orc.fp16_to_fp32(h).view(np.uint32)) == str(golden["f16_dec_all_sha"])


@pytest.mark.parametrize("name,ms,hd,base", [("rt_2048_64_1e4", 2048, 64, 10000.0),
                                             ("rt_32800_64_5e5", 32800, 64, 500000.0)])
def test_rope_tables_digest(golden, orc, name, ms, hd, base):
    c, s = orc.rope_tables(ms, hd, base)
    np.testing.assert_array_equal(np.stack([c[:4 * hd // 2], s[:4 * hd // 2]]),
                                  golden[name + "_head"])
    assert sha(c) == str(golden[name + "_cos_sha"])
    assert sha(s) == str(golden[name + "_sin_sha"])


@pytest.mark.parametrize("rope_type", [0, 1])
def test_rope_apply(golden, orc, rope_type):
    c, s = orc.rope_tables(256, 64, 10000.0)
    q, k = golden["rope_q_in"].copy(), golden["rope_k_in"].copy()
    orc.port().orc_rope(q, k, 64, 32, 4, np.ascontiguousarray(c[255 * 32:256 * 32]),
                        np.ascontiguousarray(s[255 * 32:256 * 32]), rope_type)
    np.testing.assert_array_equal(q.view(np.uint32),
                                  golden[f"rope_q_out_t{rope_type}"].view(np.uint32))
    np.testing.assert_array_equal(k.view(np.uint32),
                                  golden[f"rope_k_out_t{rope_type}"].view(np.uint32))


@pytest.mark.parametrize("pos", [0, 1, 17, 63])
def test_decode_layer_small(golden, orc, pos):
    H, Hk, hd, ms = 8, 2, 64, 64
    c = orc.cfg(H, Hk, hd, ms)
    ct, st = orc.rope_tables(ms, hd, 10000.0)
    assert sha(ct) == str(golden["dsm_cos_sha"])
    kc, vc = golden["dsm_kc0"].copy(), golden["dsm_vc0"].copy()
    out, _, _ = orc.attn_decode(c, kc.ravel(), vc.ravel(), pos, golden[f"dsm_p{pos}_q"],
                                golden[f"dsm_p{pos}_k"], golden[f"dsm_p{pos}_v"], ct, st)
    np.testing.assert_array_equal(kc[pos], golden[f"dsm_p{pos}_krow"])
    np.testing.assert_array_equal(vc[pos], golden[f"dsm_p{pos}_vrow"])
    np.testing.assert_array_equal(out.view(np.uint32),
                                  golden[f"dsm_p{pos}_out"].view(np.uint32))
    # only row `pos` changed
    mask = np.ones(ms, bool)
    mask[pos] = False
    np.testing.assert_array_equal(kc[mask], golden["dsm_kc0"][mask])


def config1_inputs():
    """TinyLlama config-1 inputs regenerated from seed 0 (digest-checked)."""
    from tests.golden.make_golden import decode_inputs
    from oracle import oracle as O
    H, Hk, hd, ms, P = 32, 4, 64, 256, 255
    rng = np.random.default_rng(0)
    x, wq, wk, wv, cache_f = decode_inputs(rng, H, Hk, hd, ms)
    kc0 = O.fp32_to_fp16(cache_f[0]).reshape(ms, Hk * hd)
    vc0 = O.fp32_to_fp16(cache_f[1]).reshape(ms, Hk * hd)
    kc0[P:] = 0
    vc0[P:] = 0
    return x, wq, wk, wv, kc0, vc0


def test_decode_config1(golden, orc):
    x, wq, wk, wv, kc0, vc0 = config1_inputs()
    assert sha(np.concatenate([x, wq.ravel(), wk.ravel(), wv.ravel()])) == \
        str(golden["c1_inputs_sha"])
    assert sha(np.stack([kc0, vc0])) == str(golden["c1_cache_sha"])
    c = orc.cfg(32, 4, 64, 256)
    ct, st = orc.rope_tables(256, 64, 10000.0)
    kc, vc = kc0.copy(), vc0.copy()
    out, _, _ = orc.attn_decode(c, kc.ravel(), vc.ravel(), 255, golden["c1_q"],
                                golden["c1_k"], golden["c1_v"], ct, st)
    np.testing.assert_array_equal(kc[255], golden["c1_krow"])
    np.testing.assert_array_equal(vc[255], golden["c1_vrow"])
    np.testing.assert_array_equal(out.view(np.uint32), golden["c1_out"].view(np.uint32))


def test_prefill_append_matches_model_forward_prefill(golden, orc):
    H, Hk, hd, ms, S0, N = 8, 2, 64, 64, 8, 16
    c = orc.cfg(H, Hk, hd, ms)
    ct, st = orc.rope_tables(ms, hd, 10000.0)
    kc, vc = golden["pf_kc0"].copy(), golden["pf_vc0"].copy()
    orc.attn_prefill(c, kc.ravel(), vc.ravel(), S0, golden["pf_q"], golden["pf_k"],
                     golden["pf_v"], ct, st)
    np.testing.assert_array_equal(kc[S0:S0 + N], golden["pf_krows"])
    np.testing.assert_array_equal(vc[S0:S0 + N], golden["pf_vrows"])


def test_prefill_outputs_match_decode_chain(golden, orc):
    H, Hk, hd, ms, S0, N = 8, 2, 64, 64, 8, 16
    c = orc.cfg(H, Hk, hd, ms)
    ct, st = orc.rope_tables(ms, hd, 10000.0)
    kc, vc = golden["pf_kc0"].copy(), golden["pf_vc0"].copy()
    out, _, _ = orc.attn_prefill(c, kc.ravel(), vc.ravel(), S0, golden["pfd_q"],
                                 golden["pfd_k"], golden["pfd_v"], ct, st)
    np.testing.assert_array_equal(out.view(np.uint32), golden["pfd_out"].view(np.uint32))
    np.testing.assert_array_equal(kc[S0:S0 + N], golden["pfd_krows"])


def test_decode_seqs_threads_equal_single(orc):
    rng = np.random.default_rng(5)
    H, Hk, hd, ms, n = 8, 2, 64, 40, 6
    c = orc.cfg(H, Hk, hd, ms)
    ct, st = orc.rope_tables(ms, hd, 10000.0)
    kv = Hk * hd
    cache = orc.fp32_to_fp16(rng.standard_normal(2 * n * ms * kv, dtype=np.float32))
    pos = rng.integers(0, ms, n).astype(np.int32)
    q = rng.standard_normal(n * H * hd, dtype=np.float32)
    k = rng.standard_normal(n * kv, dtype=np.float32)
    v = rng.standard_normal(n * kv, dtype=np.float32)
    outs = []
    for th in (1, 3):
        kc, vc = cache[:n * ms * kv].copy(), cache[n * ms * kv:].copy()
        outs.append(orc.attn_decode_seqs(c, kc, vc, ms * kv, pos, q, k, v, ct, st, th))
    np.testing.assert_array_equal(outs[0], outs[1])


@pytest.mark.skipif(not __import__("oracle.oracle", fromlist=["x"]).ref_available(),
                    reason="oracle/_ref (the reference compiled here) is absent")
@pytest.mark.parametrize("H,Hk,hd", [(32, 4, 64), (32, 8, 128), (16, 2, 128)])
def test_port_equals_genuine_reference_live(orc, H, Hk, hd):
    # head_dim 128 (model.c:856 takes any hd <= 256) pins the restatement at
    # the second head size the CUDA kernels support
    rng = np.random.default_rng(7 + hd + Hk)
    ms, n = 300, 4
    c = orc.cfg(H, Hk, hd, ms)
    ct, st = orc.rope_tables(ms, hd, 10000.0)
    ct2 = np.empty_like(ct)
    st2 = np.empty_like(st)
    orc.ref().ref_rope_tables(ct2, st2, ms, hd, 10000.0)
    np.testing.assert_array_equal(ct, ct2)
    kv = Hk * hd
    cache = orc.fp32_to_fp16(rng.standard_normal(2 * n * ms * kv, dtype=np.float32))
    pos = np.array([0, 7, 150, 299], np.int32)
    q = rng.standard_normal(n * H * hd, dtype=np.float32) * 3
    k = rng.standard_normal(n * kv, dtype=np.float32) * 3
    v = rng.standard_normal(n * kv, dtype=np.float32)
    res = []
    for use_ref in (False, True):
        kc, vc = cache[:n * ms * kv].copy(), cache[n * ms * kv:].copy()
        out = orc.attn_decode_seqs(c, kc, vc, ms * kv, pos, q, k, v, ct, st, 2,
                                   use_ref=use_ref)
        res.append((out, kc, vc))
    np.testing.assert_array_equal(res[0][0].view(np.uint32), res[1][0].view(np.uint32))
    np.testing.assert_array_equal(res[0][1], res[1][1])
    np.testing.assert_array_equal(res[0][2], res[1][2])
    # random bit patterns through both encoders
    bits = rng.integers(0, 1 << 32, 200000, dtype=np.uint64).astype(np.uint32)
    f = bits.view(np.float32)
    want = np.empty(f.size, np.uint16)
    orc.ref().ref_fp32_to_fp16_array(f, want, f.size)
    np.testing.assert_array_equal(orc.fp32_to_fp16(f), want)
    h = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    dec = np.empty(65536, np.float32)
    orc.ref().ref_fp16_to_fp32_array(h, dec, 65536)
    np.testing.assert_array_equal(orc.fp16_to_fp32(h).view(np.uint32), dec.view(np.uint32))


@pytest.mark.skipif(not __import__("oracle.oracle", fromlist=["x"]).ref_available(),
                    reason="oracle/_ref (the reference compiled here) is absent")
@pytest.mark.parametrize("hd,rope_type", [(64, 0), (64, 1), (128, 0), (128, 1)])
def test_rope_port_equals_genuine_reference(orc, hd, rope_type):
    # the restated rotation against picolm's own rope() (tensor.c:533-601),
    # both pairings, at both supported head sizes, bit for bit
    rng = np.random.default_rng(hd + rope_type)
    H, Hk, ms = 8, 2, 64
    ct, st = orc.rope_tables(ms, hd, 10000.0)
    half = hd // 2
    for pos in (0, 1, 37, 63):
        q = rng.standard_normal(H * hd, dtype=np.float32) * 3
        k = rng.standard_normal(Hk * hd, dtype=np.float32) * 3
        cs = np.ascontiguousarray(ct[pos * half:(pos + 1) * half])
        sn = np.ascontiguousarray(st[pos * half:(pos + 1) * half])
        q1, k1, q2, k2 = q.copy(), k.copy(), q.copy(), k.copy()
        orc.port().orc_rope(q1, k1, hd, H, Hk, cs, sn, rope_type)
        orc.ref().rope(q2, k2, hd, H, Hk, cs, sn, rope_type)
        np.testing.assert_array_equal(q1.view(np.uint32), q2.view(np.uint32))
        np.testing.assert_array_equal(k1.view(np.uint32), k2.view(np.uint32))


# ---- projections around the attention path (matmul per GGUF type, rmsnorm)
@pytest.mark.parametrize("name", ["f32", "f16", "q8_0", "q4_k", "q6_k"])
def test_matmul_port_equals_golden(golden, orc, name):
    from tests.util import GGUF_TYPES
    w, x, want = golden[f"proj_{name}_w"], golden[f"proj_{name}_x"], golden[f"proj_{name}_out"]
    got = orc.matmul(w, x, x.size, want.size, GGUF_TYPES[name])
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("size", [2048, 61])
def test_rmsnorm_port_equals_golden(golden, orc, size):
    x, w, want = golden[f"rms{size}_x"], golden[f"rms{size}_w"], golden[f"rms{size}_out"]
    got = orc.rmsnorm(x, w, 1e-5)
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.skipif(not __import__("oracle.oracle", fromlist=["x"]).ref_available(),
                    reason="oracle/_ref (the reference compiled here) is absent")
@pytest.mark.parametrize("name", ["f32", "f16", "q8_0", "q4_k", "q6_k"])
def test_matmul_port_equals_genuine_reference(orc, name):
    # TinyLlama's projection shapes: 256 rows of 2048 inputs (Wk) and 2048
    # inputs of a 2048-wide Wo slice, fresh weights, bit for bit
    from tests.util import GGUF_TYPES, random_gguf
    t = GGUF_TYPES[name]
    rng = np.random.default_rng(100 + t)
    for rows, n in ((256, 2048), (40, 4096)):
        w = random_gguf(rng, t, rows, n)
        assert w.shape[1] == orc.row_bytes(t, n)
        x = rng.standard_normal(n, dtype=np.float32)
        a = orc.matmul(w, x, n, rows, t)
        b = orc.matmul(w, x, n, rows, t, use_ref=True)
        np.testing.assert_array_equal(a.view(np.uint32), b.view(np.uint32))
