"""The attention sub-block with its projections on the device, through the C
ABI, against the oracle chain of picolm's own steps:

  rmsnorm -> matmul Q, K, V (+ biases) -> QK-norm -> RoPE, FP16 append,
  attention -> matmul O (+ bias) -> residual add        (model.c:779-897)

The projections sum in another order than the CPU, so their outputs agree
with picolm's to FP32 rounding (checked against 1e-4 of the output scale);
the residual stream after the block is held to the attention tolerance
(max-abs 2e-3, rel 1e-2), and the appended FP16 KV rows must equal the
oracle's or sit one unit away where the FP32 value is at a rounding
boundary (assert_kv_near).
"""
import numpy as np
import pytest

import picolm_b200 as pb
from oracle import oracle as O
from tests.util import (GGUF_F16, GGUF_F32, GGUF_Q4_K, GGUF_Q6_K, GGUF_Q8_0, GGUF_TYPES,
                        assert_attn_close, assert_kv_near, oracle_out, oracle_qkv,
                        random_cache, random_gguf, random_layer, upload_layer)

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _built():
    from picolm_b200 import build
    build.build()


def _close_proj(got, want, what):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    tol = 1e-4 * np.abs(want).max() + 1e-6
    err = np.abs(got - want).max()
    assert err <= tol, f"{what}: max err {err:.3e} > {tol:.3e}"


@pytest.mark.parametrize("name", list(GGUF_TYPES))
def test_projection_vs_oracle(name):
    # every projection of a layer whose four weights have this type, on 1, 5
    # and 13 input rows (13 > the 8 rows a CTA stages: two row chunks), 20
    # (the mma.sync path for Q4_K, Q8_0 and F16: 16-row tiles), 24, 40 and
    # 64 (the skinny tcgen05 GEMM over the dequantised weights, weights as
    # the A operand, K split over CTAs and the partials summed in order), 65
    # and 200 (gemm_hilo_kernel: one ragged 128-row tile, and a ragged
    # second one)
    t = GGUF_TYPES[name]
    rng = np.random.default_rng(40 + t)
    H, Hk, hd, dim = 8, 2, 64, 768
    L = random_layer(rng, H, Hk, hd, dim, types=(t,) * 4, bias=True)
    shapes = [(H * hd, dim), (Hk * hd, dim), (Hk * hd, dim), (dim, H * hd)]
    biases = [L["bq"], L["bk"], L["bv"], L["bo"]]
    with pb.Attn(1, H, Hk, 64, head_dim=hd) as at:
        upload_layer(at, 0, L)
        for which, (rows, n) in enumerate(shapes):
            for m in (1, 5, 13, 20, 24, 40, 64, 65, 200):
                x = rng.standard_normal((m, n), dtype=np.float32)
                got = at.proj(0, which, x, rows)
                for i in range(m):
                    want = O.matmul(L["w"][which], x[i], n, rows, t) + biases[which]
                    _close_proj(got[i], want, f"{name} W{which} m{m} row {i}")


@pytest.mark.parametrize("which", [0, 3])
def test_projection_gemm_many_tiles(which):
    # TinyLlama-shaped Q4_K weights over 1500 input rows: 12 x 16 = 192
    # output tiles of 128 x 128, more CTAs than the 148 SMs (a second round),
    # and a ragged last row tile; every row against the oracle
    import os
    from concurrent.futures import ThreadPoolExecutor
    rng = np.random.default_rng(77 + which)
    H, Hk, hd, dim = 32, 4, 64, 2048
    L = random_layer(rng, H, Hk, hd, dim, types=(GGUF_Q4_K,) * 4, bias=True)
    rows, n = [(H * hd, dim), (Hk * hd, dim), (Hk * hd, dim), (dim, H * hd)][which]
    bias = [L["bq"], L["bk"], L["bv"], L["bo"]][which]
    m = 1500
    x = rng.standard_normal((m, n), dtype=np.float32)
    with pb.Attn(1, H, Hk, 64, head_dim=hd) as at:
        upload_layer(at, 0, L)
        got = at.proj(0, which, x, rows)

    def one(i):
        return O.matmul(L["w"][which], x[i], n, rows, GGUF_Q4_K) + bias

    with ThreadPoolExecutor(os.cpu_count() or 4) as ex:
        want = list(ex.map(one, range(m)))
    for i in range(m):
        _close_proj(got[i], want[i], f"W{which} row {i}")


@pytest.mark.parametrize("dim", [128, 2048])
def test_projection_skinny_split_and_unsplit(dim):
    # the skinny GEMM (24-64 input rows, weights as the A operand): with 128
    # inputs a tile has two k-steps and is not split (one CTA, direct
    # epilogue); with 2048 the k-steps of a tile are split over a cluster
    # and reduced through distributed shared memory, in split order, so two
    # identical calls give identical bits
    rng = np.random.default_rng(91 + dim)
    H, Hk, hd = (2, 2, 64) if dim == 128 else (32, 4, 64)
    t = GGUF_Q8_0 if dim == 128 else GGUF_Q4_K  # Q4_K blocks span 256 inputs
    L = random_layer(rng, H, Hk, hd, dim, types=(t,) * 4, bias=True)
    shapes = [(H * hd, dim), (Hk * hd, dim), (Hk * hd, dim), (dim, H * hd)]
    biases = [L["bq"], L["bk"], L["bv"], L["bo"]]
    with pb.Attn(1, H, Hk, 64, head_dim=hd) as at:
        upload_layer(at, 0, L)
        for which in (0, 3):
            rows, n = shapes[which]
            for m in (24, 37, 64):
                x = rng.standard_normal((m, n), dtype=np.float32)
                got = at.proj(0, which, x, rows)
                again = at.proj(0, which, x, rows)
                np.testing.assert_array_equal(got.view(np.uint32), again.view(np.uint32))
                for i in range(m):
                    want = O.matmul(L["w"][which], x[i], n, rows, t) + biases[which]
                    _close_proj(got[i], want, f"dim {dim} W{which} m{m} row {i}")


def test_projection_wide_input():
    # head_dim 128 x 32 heads: Wo takes 4096 inputs (16 KB a staged row)
    rng = np.random.default_rng(3)
    H, Hk, hd, dim = 32, 8, 128, 512
    L = random_layer(rng, H, Hk, hd, dim, types=(GGUF_Q8_0, GGUF_F16, GGUF_Q6_K, GGUF_Q4_K))
    with pb.Attn(1, H, Hk, 64, head_dim=hd) as at:
        upload_layer(at, 0, L)
        x = rng.standard_normal((9, H * hd), dtype=np.float32)
        got = at.proj(0, 3, x, dim)
        for i in range(9):
            _close_proj(got[i], O.matmul(L["w"][3], x[i], H * hd, dim, GGUF_Q4_K), f"Wo row {i}")


CASES = [
    # H, Hk, hd, dim, types (q, k, v, o), bias, qk_norm, rope_type
    (32, 4, 64, 2048, (GGUF_Q4_K,) * 4, False, False, 0),            # TinyLlama, Q4_K
    (16, 2, 128, 1024, (GGUF_Q6_K, GGUF_Q8_0, GGUF_F16, GGUF_F32), True, True, 1),  # Qwen3-like
    (8, 8, 64, 512, (GGUF_Q8_0, GGUF_Q4_K, GGUF_Q6_K, GGUF_Q4_K), True, False, 0),
]


@pytest.mark.parametrize("H,Hk,hd,dim,types,bias,qk_norm,rope_type", CASES)
def test_block_decode_vs_oracle(H, Hk, hd, dim, types, bias, qk_norm, rope_type):
    rng = np.random.default_rng(H + Hk + hd + dim)
    ms, layer, n_layers = 320, 1, 2
    kv = Hk * hd
    L = random_layer(rng, H, Hk, hd, dim, types=types, bias=bias, qk_norm=qk_norm)
    tables = O.rope_tables(ms, hd, 10000.0)
    pos0 = [0, 1, 63, 200]
    n = len(pos0)
    caches = [[random_cache(rng, ms, kv), random_cache(rng, ms, kv)] for _ in range(n)]
    with pb.Attn(n_layers, H, Hk, ms, rope_type=rope_type, n_seqs=n, head_dim=hd) as at:
        upload_layer(at, layer, L)
        for s in range(n):
            at.kv_upload(s, layer, 0, *caches[s])
        seqs = np.arange(n, dtype=np.int32)
        rows_dev, rows_want = [], []
        for step in range(2):   # the second step attends the row the first appended
            pos = np.array(pos0, np.int32) + step
            x = rng.standard_normal((n, dim), dtype=np.float32)
            got = at.block_decode(layer, seqs, pos, x)
            for s in range(n):
                q, k, v = oracle_qkv(H, Hk, hd, L, x[s])
                c = O.cfg(H, Hk, hd, ms, rope_type)
                kc, vc = caches[s]
                kc2, vc2 = kc.copy(), vc.copy()
                att, _, _ = O.attn_decode(c, kc2.ravel(), vc2.ravel(), int(pos[s]), q, k, v,
                                          *tables)
                want = oracle_out(H, hd, L, x[s], att)
                assert_attn_close(got[s], want, f"step {step} seq {s} pos {pos[s]}")
                gk, gv = at.kv_download(s, layer, 0, ms)
                p = int(pos[s])
                assert_kv_near(gk[p], kc2[p], f"k row {p}", max_frac=1.0)
                assert_kv_near(gv[p], vc2[p], f"v row {p}", max_frac=1.0)
                rows_dev += [gk[p], gv[p]]
                rows_want += [kc2[p], vc2[p]]
                np.testing.assert_array_equal(np.delete(gk, p, 0), np.delete(kc, p, 0))
                # carry the device's rows forward so the next step's oracle
                # attends exactly what the device holds
                caches[s] = [gk.copy(), gv.copy()]
    assert_kv_near(np.stack(rows_dev), np.stack(rows_want), "appended k and v rows")


@pytest.mark.parametrize("types", [(GGUF_Q4_K,) * 4, (GGUF_Q8_0, GGUF_F16, GGUF_Q8_0, GGUF_F16)])
def test_block_decode_many_sequences(types):
    """24 sequences: the projections take the skinny tcgen05 GEMM (24-64
    input rows: weights as the A operand, K split over a cluster)."""
    rng = np.random.default_rng(sum(types))
    H, Hk, hd, dim, ms, n = 32, 4, 64, 2048, 96, 24
    kv = Hk * hd
    L = random_layer(rng, H, Hk, hd, dim, types=types, bias=True)
    tables = O.rope_tables(ms, hd, 10000.0)
    caches = [(random_cache(rng, ms, kv), random_cache(rng, ms, kv)) for _ in range(n)]
    pos = rng.integers(0, ms, n).astype(np.int32)
    x = rng.standard_normal((n, dim), dtype=np.float32)
    with pb.Attn(1, H, Hk, ms, n_seqs=n) as at:
        upload_layer(at, 0, L)
        for s_, (kc, vc) in enumerate(caches):
            at.kv_upload(s_, 0, 0, kc, vc)
        got = at.block_decode(0, np.arange(n, dtype=np.int32), pos, x)
        kv_dev = [at.kv_download(s_, 0, 0, ms) for s_ in range(n)]
    rows_dev, rows_want = [], []
    for s_ in range(n):
        q, k, v = oracle_qkv(H, Hk, hd, L, x[s_])
        kc2, vc2 = caches[s_][0].copy(), caches[s_][1].copy()
        att, _, _ = O.attn_decode(O.cfg(H, Hk, hd, ms), kc2.ravel(), vc2.ravel(), int(pos[s_]),
                                  q, k, v, *tables)
        assert_attn_close(got[s_], oracle_out(H, hd, L, x[s_], att), f"seq {s_}")
        p_ = int(pos[s_])
        rows_dev += [kv_dev[s_][0][p_], kv_dev[s_][1][p_]]
        rows_want += [kc2[p_], vc2[p_]]
    assert_kv_near(np.stack(rows_dev), np.stack(rows_want), "appended k and v rows")


@pytest.mark.parametrize("H,Hk,hd,dim,types,bias,qk_norm,rope_type", CASES[:2])
def test_block_prefill_vs_oracle(H, Hk, hd, dim, types, bias, qk_norm, rope_type):
    """(1) The module's prefill attention on the oracle's own q, k, v
    (pl_attn_prefill) against the oracle's: the attention tolerance.
    (2) The appended K/V rows of the block: assert_kv_near.  (3) The block's
    output against the oracle's output projection and residual applied to
    the oracle attention (the restated model.c:848-892 loop) of the oracle's
    rotated q over the K/V rows the device holds.  Using the device's rows
    in (3) keeps out the effect of FP16 words that the two FP32 projections
    round to neighbouring values: with P in FP16 such a word can move a
    near-tied prefill output by about 1e-3."""
    rng = np.random.default_rng(7 * H + hd)
    start, n_tok = 5, 130
    ms = start + n_tok + 3
    kv = Hk * hd
    L = random_layer(rng, H, Hk, hd, dim, types=types, bias=bias, qk_norm=qk_norm)
    tables = O.rope_tables(ms, hd, 10000.0)
    kc = np.zeros((ms, kv), np.uint16)
    vc = np.zeros((ms, kv), np.uint16)
    kc[:start] = random_cache(rng, start, kv)
    vc[:start] = random_cache(rng, start, kv)
    x = rng.standard_normal((n_tok, dim), dtype=np.float32)
    qkv = [oracle_qkv(H, Hk, hd, L, x[i]) for i in range(n_tok)]
    q = np.stack([a[0] for a in qkv])
    k = np.stack([a[1] for a in qkv])
    v = np.stack([a[2] for a in qkv])
    with pb.Attn(1, H, Hk, ms, rope_type=rope_type, head_dim=hd) as at:
        upload_layer(at, 0, L)
        at.kv_upload(0, 0, 0, kc, vc)
        att_dev = at.prefill(0, 0, start, q, k, v)     # the module's attention, oracle inputs
        at.kv_upload(0, 0, 0, kc, vc)
        got = at.block_prefill(0, 0, start, x)
        gk, gv = at.kv_download(0, 0, 0, ms)
    c = O.cfg(H, Hk, hd, ms, rope_type)
    kc2, vc2 = kc.copy(), vc.copy()
    att, q_rot, _ = O.attn_prefill(c, kc2.ravel(), vc2.ravel(), start, q, k, v, *tables)
    assert_attn_close(att_dev, att, "prefill attention on the oracle's q, k, v")
    assert_kv_near(gk[start:start + n_tok], kc2[start:start + n_tok], "k rows")
    assert_kv_near(gv[start:start + n_tok], vc2[start:start + n_tok], "v rows")
    np.testing.assert_array_equal(gk[:start], kc[:start])
    gkf, gvf = np.ascontiguousarray(gk.ravel()), np.ascontiguousarray(gv.ravel())
    for i in range(n_tok):
        att_i = np.empty(H * hd, np.float32)
        O.port().orc_attn_core(O.ctypes_ref(c), gkf, gvf, start + i,
                               np.ascontiguousarray(q_rot[i]), att_i)
        assert_attn_close(got[i], oracle_out(H, hd, L, x[i], att_i), f"block row {i}")


def test_block_dev_equals_host():
    # the device-pointer entry points run the same launches: bit-identical
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(11)
    H, Hk, hd, dim, ms, n = 32, 4, 64, 2048, 256, 3
    L = random_layer(rng, H, Hk, hd, dim)
    x = rng.standard_normal((n, dim), dtype=np.float32)
    xp = rng.standard_normal((40, dim), dtype=np.float32)
    pos = np.array([10, 100, 255], np.int32)
    seqs = np.arange(n, dtype=np.int32)
    res = []
    for dev in (False, True):
        with pb.Attn(1, H, Hk, ms, n_seqs=n) as at:
            upload_layer(at, 0, L)
            if dev:
                d = torch.device("cuda", 0)
                tx = torch.from_numpy(x).to(d)
                tp = torch.from_numpy(xp).to(d)
                ts, tq = torch.from_numpy(seqs).to(d), torch.from_numpy(pos).to(d)
                st = torch.cuda.current_stream(d).cuda_stream
                at.block_prefill_dev(1, 0, 0, 40, tp.data_ptr(), st)
                at.block_decode_dev(0, n, ts.data_ptr(), tq.data_ptr(), 255, tx.data_ptr(), st)
                torch.cuda.synchronize()
                a, b = tx.cpu().numpy(), tp.cpu().numpy()
            else:
                b = at.block_prefill(1, 0, 0, xp)
                a = at.block_decode(0, seqs, pos, x)
            res.append((a, b, at.kv_download(1, 0, 0, 41)))
    np.testing.assert_array_equal(res[0][0].view(np.uint32), res[1][0].view(np.uint32))
    np.testing.assert_array_equal(res[0][1].view(np.uint32), res[1][1].view(np.uint32))
    np.testing.assert_array_equal(res[0][2][0], res[1][2][0])


def test_set_layer_errors():
    rng = np.random.default_rng(5)
    H, Hk, hd, dim = 8, 2, 64, 512
    L = random_layer(rng, H, Hk, hd, dim)
    with pb.Attn(2, H, Hk, 64) as at:
        x = rng.standard_normal((1, dim), dtype=np.float32)
        with pytest.raises(pb.PlAttnError) as e:      # no weights for the layer yet
            at.block_decode(0, [0], [3], x)
        assert e.value.rc == pb.PL_ESTATE
        w = L["w"]
        with pytest.raises(pb.PlAttnError) as e:      # Q4_0 (type 2) is not taken
            at.set_layer(0, dim, w[0], 2, w[1], GGUF_Q4_K, w[2], GGUF_Q4_K, w[3], GGUF_Q4_K)
        assert e.value.rc == pb.PL_EUNSUPPORTED
        with pytest.raises(pb.PlAttnError) as e:      # dim not a multiple of the block
            at.set_layer(0, 500, w[0], GGUF_Q4_K, w[1], GGUF_Q4_K, w[2], GGUF_Q4_K, w[3],
                         GGUF_Q4_K)
        assert e.value.rc == pb.PL_EUNSUPPORTED
        with pytest.raises(pb.PlAttnError) as e:      # q_norm without k_norm
            at.set_layer(0, dim, *sum(([a, GGUF_Q4_K] for a in w), []),
                         q_norm=np.ones(hd, np.float32))
        assert e.value.rc == pb.PL_EARG
        upload_layer(at, 1, L)
        with pytest.raises(pb.PlAttnError) as e:      # position past max_seq
            at.block_decode(1, [0], [64], x)
        assert e.value.rc == pb.PL_EARG
        out = at.block_decode(1, [0], [0], x)           # the module is still usable
        assert np.isfinite(out).all()
        assert not np.array_equal(out, x)
