"""One module context over several devices (pl_attn_init_devices), GPU.

Both layouts are checked against the oracle's restatement of
picolm/model.c:848-892 (decode) and 1039-1089 (prefill):
* PL_SPLIT_KV: each slot's cache rows in 512-position blocks spread over
  the devices; a decode merges the devices' partials with a log-sum-exp
  combine on the first device, a prefill gathers the earlier rows there and
  returns the new rows to their owners.  Positions are chosen so every
  device holds rows and blocks are crossed; the whole cache is downloaded
  (through the same block map) and compared bit for bit.
* PL_SPLIT_SEQS: slots spread over the devices, a batch in shuffled slot
  order split by owner.

A device id may repeat: [0, 0] runs the whole fan-out (staging per context,
events, the combine, the gather and scatter copies) on one GPU, so these
run on a one-GPU box; on a box with more GPUs the same tests also run over
distinct devices, where the combine and the gathers cross NVLink.
"""
import numpy as np
import pytest

import picolm_b200 as pb
from oracle import oracle as O
from tests.util import assert_attn_close, random_cache

pytestmark = pytest.mark.gpu


def _device_sets():
    import torch
    sets = [[0, 0], [0, 0, 0]]
    n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    if n >= 2:
        sets.append([0, 1])
    if n >= 4:
        sets.append([0, 1, 2, 3])
    return sets


@pytest.fixture(scope="module", autouse=True)
def _built():
    from picolm_b200 import build
    build.build()


@pytest.mark.parametrize("devices", _device_sets(), ids=lambda d: "dev" + "".join(map(str, d)))
@pytest.mark.parametrize("hd,H,Hk", [(64, 32, 8), (128, 16, 4)])
def test_kv_split_decode_and_prefill_vs_oracle(devices, hd, H, Hk):
    rng = np.random.default_rng(31 + len(devices) + hd)
    L, n_seqs, ms, theta = 2, 2, 2600, 500000.0
    kv = Hk * hd
    tables = O.rope_tables(ms, hd, theta)
    c = O.cfg(H, Hk, hd, ms)
    caches = {}
    with pb.Attn(L, H, Hk, ms, rope_base=theta, n_seqs=n_seqs, head_dim=hd, devices=devices,
                 split=pb.PL_SPLIT_KV) as at:
        # slot 1, layer 1: 1900 rows uploaded, then decode steps across blocks
        kc = np.zeros((ms, kv), np.uint16)
        vc = np.zeros((ms, kv), np.uint16)
        kc[:1900] = random_cache(rng, 1900, kv)
        vc[:1900] = random_cache(rng, 1900, kv)
        at.kv_upload(1, 1, 0, kc[:1900], vc[:1900])
        for pos in (1900, 1901, 2047, 2048):  # 2048 opens a new block
            if pos == 2047:
                kc[1902:2047] = random_cache(rng, 145, kv)
                vc[1902:2047] = random_cache(rng, 145, kv)
                at.kv_upload(1, 1, 1902, kc[1902:2047], vc[1902:2047])
            q = rng.standard_normal(H * hd, dtype=np.float32)
            k = rng.standard_normal(kv, dtype=np.float32)
            v = rng.standard_normal(kv, dtype=np.float32)
            got = at.decode(1, 1, pos, q, k, v)
            want, _, _ = O.attn_decode(c, kc.ravel(), vc.ravel(), pos, q, k, v, *tables)
            assert_attn_close(got, want, f"KV-split decode at {pos}")
        caches[(1, 1)] = (kc, vc)
        # slot 0, layer 0: a prefill over rows of every device after 700 cached
        kc0 = np.zeros((ms, kv), np.uint16)
        vc0 = np.zeros((ms, kv), np.uint16)
        kc0[:700] = random_cache(rng, 700, kv)
        vc0[:700] = random_cache(rng, 700, kv)
        at.kv_upload(0, 0, 0, kc0[:700], vc0[:700])
        n_tok = 1100
        qp = rng.standard_normal((n_tok, H * hd), dtype=np.float32)
        kp = rng.standard_normal((n_tok, kv), dtype=np.float32)
        vp = rng.standard_normal((n_tok, kv), dtype=np.float32)
        got = at.prefill(0, 0, 700, qp, kp, vp)
        want, _, _ = O.attn_prefill(c, kc0.ravel(), vc0.ravel(), 700, qp, kp, vp, *tables)
        assert_attn_close(got, want, "KV-split prefill")
        # and a decode right after it, attending the rows the prefill scattered
        q = rng.standard_normal(H * hd, dtype=np.float32)
        k = rng.standard_normal(kv, dtype=np.float32)
        v = rng.standard_normal(kv, dtype=np.float32)
        got = at.decode(0, 0, 1800, q, k, v)
        want, _, _ = O.attn_decode(c, kc0.ravel(), vc0.ravel(), 1800, q, k, v, *tables)
        assert_attn_close(got, want, "KV-split decode after prefill")
        caches[(0, 0)] = (kc0, vc0)
        for (s, l), (kw, vw) in caches.items():
            gk, gv = at.kv_download(s, l, 0, ms)
            np.testing.assert_array_equal(gk, kw, f"slot {s} layer {l} K")
            np.testing.assert_array_equal(gv, vw, f"slot {s} layer {l} V")
        assert at.status() == pb.PL_OK
        # single-device entry points are refused on a multi-device context
        with pytest.raises(pb.PlAttnError) as ei:
            at.decode_batch_dev(0, 1, 0, 0, 0, 0, 0, 0, 0)
        assert ei.value.rc == pb.PL_EUNSUPPORTED


@pytest.mark.parametrize("devices", _device_sets(), ids=lambda d: "dev" + "".join(map(str, d)))
def test_seq_split_batch_vs_oracle(devices):
    rng = np.random.default_rng(41 + len(devices))
    H, Hk, hd, ms, n = 32, 4, 64, 700, 7
    kv = Hk * hd
    tables = O.rope_tables(ms, hd, 10000.0)
    c = O.cfg(H, Hk, hd, ms)
    kc = np.zeros((n, ms, kv), np.uint16)
    vc = np.zeros((n, ms, kv), np.uint16)
    lengths = rng.integers(1, ms - 200, n)
    with pb.Attn(1, H, Hk, ms, n_seqs=n, devices=devices, split=pb.PL_SPLIT_SEQS) as at:
        for s in range(n):
            kc[s, :lengths[s]] = random_cache(rng, int(lengths[s]), kv)
            vc[s, :lengths[s]] = random_cache(rng, int(lengths[s]), kv)
            at.kv_upload(s, 0, 0, kc[s, :lengths[s]], vc[s, :lengths[s]])
        order = rng.permutation(n).astype(np.int32)
        pos = lengths[order].astype(np.int32)
        q = rng.standard_normal((n, H * hd), dtype=np.float32)
        k = rng.standard_normal((n, kv), dtype=np.float32)
        v = rng.standard_normal((n, kv), dtype=np.float32)
        got = at.decode_batch(0, order, pos, q, k, v)
        for j, s in enumerate(order):
            want, _, _ = O.attn_decode(c, kc[s].ravel(), vc[s].ravel(), int(pos[j]), q[j], k[j],
                                       v[j], *tables)
            assert_attn_close(got[j], want, f"slot {s}")
        # a prefill on the last slot (owned by the last device)
        s = n - 1
        p0 = int(lengths[s]) + 1
        qp = rng.standard_normal((150, H * hd), dtype=np.float32)
        kp = rng.standard_normal((150, kv), dtype=np.float32)
        vp = rng.standard_normal((150, kv), dtype=np.float32)
        got = at.prefill(s, 0, p0, qp, kp, vp)
        want, _, _ = O.attn_prefill(c, kc[s].ravel(), vc[s].ravel(), p0, qp, kp, vp, *tables)
        assert_attn_close(got, want, "prefill on the last device")
        for s in range(n):
            gk, gv = at.kv_download(s, 0, 0, ms)
            np.testing.assert_array_equal(gk, kc[s], f"slot {s} K")
            np.testing.assert_array_equal(gv, vc[s], f"slot {s} V")
