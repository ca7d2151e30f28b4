"""Parity at the shapes the bench times, and FP16 special values on the device.

* Config 5 at its full length: one sequence of 32768 cached rows, 32 query
  heads over 8 KV heads, head_dim 64, RoPE theta 5e5, two layers x two decode
  steps, every head of every output checked against the oracle's restatement
  of picolm/model.c:848-892, and the appended K/V rows bit for bit.  At this
  length the decode kernel splits the sequence over every CTA of the grid and
  the merge takes its single-round-trip path (148 segments in flight).
* Config 4 at its full shape: 64 sequences x 2048 cached rows, 32/4 heads,
  two steps through the device-pointer entry point the bench times, every
  sequence checked and the appended rows bit-exact.
* picolm's FP32 -> FP16 encoder (quant.c:41-78: ties away from zero, FP32
  subnormals to signed zero, overflow to infinity, NaN to sign|0x7E00, FP16
  subnormals rounded half up) on the device: special values fed as V rows
  (stored without rotation) and, where RoPE at position 0 leaves them
  unchanged, as K rows, through the decode kernel's append and the prefill
  prologue's append.  The words are compared with the genuine reference's
  encoder (golden fixture) and with the oracle.
"""
import os

import numpy as np
import pytest

import picolm_b200 as pb
from oracle import oracle as O
from tests.util import assert_attn_close, random_cache

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _built():
    from picolm_b200 import build
    build.build()


def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda")


def test_config5_full_length_vs_oracle():
    import torch
    H, Hk, hd, ctx, theta = 32, 8, 64, 32768, 500000.0
    L, steps = 2, 2
    ms = ctx + steps
    kv = Hk * hd
    rng = np.random.default_rng(4)
    tables = O.rope_tables(ms, hd, theta)
    c = O.cfg(H, Hk, hd, ms)
    with pb.Attn(L, H, Hk, ms, rope_base=theta) as at:
        caches = []
        for l in range(L):
            kc = np.zeros((ms, kv), np.uint16)
            vc = np.zeros((ms, kv), np.uint16)
            kc[:ctx] = random_cache(rng, ctx, kv)
            vc[:ctx] = random_cache(rng, ctx, kv)
            at.kv_upload(0, l, 0, kc[:ctx], vc[:ctx])
            caches.append((kc, vc))
        seq = _dev(np.zeros(1, np.int32))
        st = torch.cuda.current_stream().cuda_stream
        for s in range(steps):
            pos = ctx + s
            posd = _dev(np.array([pos], np.int32))
            for l in range(L):
                q = rng.standard_normal(H * hd, dtype=np.float32)
                k = rng.standard_normal(kv, dtype=np.float32)
                v = rng.standard_normal(kv, dtype=np.float32)
                qd, kd, vd = _dev(q), _dev(k), _dev(v)
                out = torch.full((H * hd,), float("nan"), device="cuda")
                # max_pos as the bench passes it (the last step's position)
                at.decode_batch_dev(l, 1, seq.data_ptr(), posd.data_ptr(), ms - 1, qd.data_ptr(),
                                    kd.data_ptr(), vd.data_ptr(), out.data_ptr(), st)
                torch.cuda.synchronize()
                kc, vc = caches[l]
                want, _, _ = O.attn_decode(c, kc.ravel(), vc.ravel(), pos, q, k, v, *tables)
                assert_attn_close(out.cpu().numpy(), want, f"config 5 step {s} layer {l}")
        for l in range(L):
            gk, gv = at.kv_download(0, l, ctx - 1, steps + 1)
            kc, vc = caches[l]
            np.testing.assert_array_equal(gk, kc[ctx - 1:ms], f"layer {l} K rows")
            np.testing.assert_array_equal(gv, vc[ctx - 1:ms], f"layer {l} V rows")


def test_config4_full_shape_vs_oracle():
    import torch
    H, Hk, hd, ctx, n = 32, 4, 64, 2048, 64
    steps = 2
    ms = ctx + 64
    kv = Hk * hd
    rng = np.random.default_rng(3)
    tables = O.rope_tables(ms, hd, 10000.0)
    c = O.cfg(H, Hk, hd, ms)
    kc = np.zeros((n, ms, kv), np.uint16)
    vc = np.zeros((n, ms, kv), np.uint16)
    with pb.Attn(1, H, Hk, ms, n_seqs=n) as at:
        for s in range(n):
            kc[s, :ctx] = random_cache(rng, ctx, kv)
            vc[s, :ctx] = random_cache(rng, ctx, kv)
            at.kv_upload(s, 0, 0, kc[s, :ctx], vc[s, :ctx])
        # the batch in a shuffled slot order, as a scheduler may hand it over
        order = rng.permutation(n).astype(np.int32)
        seqs = _dev(order)
        st = torch.cuda.current_stream().cuda_stream
        kf, vf = kc.reshape(-1), vc.reshape(-1)
        for s in range(steps):
            pos = np.full(n, ctx + s, np.int32)
            q = rng.standard_normal((n, H * hd), dtype=np.float32)
            k = rng.standard_normal((n, kv), dtype=np.float32)
            v = rng.standard_normal((n, kv), dtype=np.float32)
            out = torch.full((n, H * hd), float("nan"), device="cuda")
            # the device copies must outlive the asynchronous call
            dpos, dq, dk, dv = _dev(pos), _dev(q), _dev(k), _dev(v)
            at.decode_batch_dev(0, n, seqs.data_ptr(), dpos.data_ptr(), ms - 1, dq.data_ptr(),
                                dk.data_ptr(), dv.data_ptr(), out.data_ptr(), st)
            torch.cuda.synchronize()
            del dpos, dq, dk, dv
            # the oracle in slot order: batch entry i is slot order[i]
            inv = np.argsort(order)
            want = O.attn_decode_seqs(c, kf, vf, ms * kv, pos, q[inv], k[inv], v[inv], *tables,
                                      n_threads=os.cpu_count() or 1)
            want = want.reshape(n, H * hd)[order]
            assert_attn_close(out.cpu().numpy(), want, f"config 4 step {s}")
        for s in range(n):
            gk, gv = at.kv_download(s, 0, ctx, steps)
            np.testing.assert_array_equal(gk, kc[s, ctx:ctx + steps], f"slot {s} K rows")
            np.testing.assert_array_equal(gv, vc[s, ctx:ctx + steps], f"slot {s} V rows")


# ------------------------------------------------------- FP16 special values
def _special_rows(golden, n_rows, width, finite_only):
    """Rows of `width` FP32 values cycling through the golden special inputs
    (FP32 subnormals, FP16 subnormal range, exact ties, overflow, +-inf, NaN
    payloads of both signs) and a sample of the tie patterns of every FP16
    exponent; finite_only drops inf and NaN (for K, which RoPE multiplies)."""
    sp = np.asarray(golden["f16_special_in"], np.float32)
    exps = np.arange(100, 143, dtype=np.uint32)
    mant = np.arange(0, 1 << 10, 37, dtype=np.uint32)
    ties = ((exps[:, None] << 23) | (mant[None, :] << 13) | 0x1000).ravel()
    ties = np.concatenate([ties, ties | 0x80000000]).view(np.float32)
    if finite_only:
        sp = sp[np.isfinite(sp)]
    # every special value first (row 0 onwards), then the tie patterns, each
    # row starting at another offset so the values meet every lane position
    vals = np.concatenate([sp, ties])
    flat = np.concatenate([sp, vals[(np.arange(n_rows * width) * 7) % vals.size]])
    return flat[:n_rows * width].reshape(n_rows, width).astype(np.float32)


@pytest.mark.parametrize("hd", [64, 128])
def test_fp16_specials_decode_append(golden, hd):
    """Specials through the decode kernel's append: V rows as given (checked
    against the genuine encoder's words too), K rows after RoPE (the same
    unfused IEEE products on both sides; at position 0, cos 1 and sin 0 keep
    finite values except that -0 comes out as +0)."""
    H, Hk, ms = 8, 2, 64
    kv = Hk * hd
    n_pos = 6
    rng = np.random.default_rng(11)
    tables = O.rope_tables(ms, hd, 10000.0)
    c = O.cfg(H, Hk, hd, ms)
    vrows = _special_rows(golden, n_pos, kv, finite_only=False)
    krows = _special_rows(golden, n_pos, kv, finite_only=True)
    kc = np.zeros((ms, kv), np.uint16)
    vc = np.zeros((ms, kv), np.uint16)
    with pb.Attn(1, H, Hk, ms, head_dim=hd) as at:
        for p in range(n_pos):
            q = rng.standard_normal(H * hd, dtype=np.float32)
            at.decode(0, 0, p, q, krows[p], vrows[p])
            O.attn_decode(c, kc.ravel(), vc.ravel(), p, q, krows[p], vrows[p], *tables)
        gk, gv = at.kv_download(0, 0, 0, n_pos)
    np.testing.assert_array_equal(gv, vc[:n_pos], "V words vs the oracle")
    np.testing.assert_array_equal(gk, kc[:n_pos], "K words vs the oracle")
    # V is stored unrotated: its words are the genuine encoder's outputs
    sp_in = np.asarray(golden["f16_special_in"], np.float32).view(np.uint32)
    sp_out = np.asarray(golden["f16_special_out"], np.uint16)
    lut = dict(zip(sp_in.tolist(), sp_out.tolist()))
    vbits = vrows.view(np.uint32)
    hits = 0
    for p in range(n_pos):
        for j in range(kv):
            b = int(vbits[p, j])
            if b in lut:
                assert int(gv[p, j]) == lut[b], (p, j, hex(b), hex(int(gv[p, j])), hex(lut[b]))
                hits += 1
    assert hits >= sp_in.size, "every special value must be checked against the reference"


@pytest.mark.parametrize("hd", [64, 128])
def test_fp16_specials_prefill_append(golden, hd):
    """Specials through the prefill prologue's append (its own encoder)."""
    H, Hk, ms = 8, 2, 160
    kv = Hk * hd
    n_tok = 130
    rng = np.random.default_rng(12)
    tables = O.rope_tables(ms, hd, 10000.0)
    c = O.cfg(H, Hk, hd, ms)
    vrows = _special_rows(golden, n_tok, kv, finite_only=False)
    krows = _special_rows(golden, n_tok, kv, finite_only=True)
    q = rng.standard_normal((n_tok, H * hd), dtype=np.float32)
    kc = np.zeros((ms, kv), np.uint16)
    vc = np.zeros((ms, kv), np.uint16)
    with pb.Attn(1, H, Hk, ms, head_dim=hd) as at:
        at.prefill(0, 0, 0, q, krows, vrows)
        gk, gv = at.kv_download(0, 0, 0, n_tok)
    O.attn_prefill(c, kc.ravel(), vc.ravel(), 0, q, krows, vrows, *tables)
    np.testing.assert_array_equal(gv, vc[:n_tok], "V words vs the oracle")
    np.testing.assert_array_equal(gk, kc[:n_tok], "K words vs the oracle")
    np.testing.assert_array_equal(gv.ravel(), O.fp32_to_fp16(vrows), "V words vs the encoder")
