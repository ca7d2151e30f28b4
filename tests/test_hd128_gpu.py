"""head_dim 128 parity: the CUDA path (through the C ABI) against the oracle.

picolm's model.c takes any head_dim up to 256 (model.c:856); the kernels
support 64 and 128, which covers the GGUF models the parser accepts in
practice (LLaMA-3 8B, Mistral 7B, Qwen2.5 7B use 128).  At 128 every row of a
Q, K or V tile is staged as two 64-element halves; the prefill runs the
tcgen05 kernel with 64-row KV tiles.  KV rows must be bit-identical to
picolm's; outputs within max-abs 2e-3 / rel 1e-2 of the oracle.
"""
import numpy as np
import pytest

import picolm_b200 as pb
from oracle import oracle as O
from tests.util import assert_attn_close, oracle_decode_layer, random_cache

pytestmark = pytest.mark.gpu

HD = 128


@pytest.fixture(scope="module", autouse=True)
def _built():
    from picolm_b200 import build
    build.build()


@pytest.mark.parametrize("H,Hk,rope_type", [(32, 8, 0), (32, 4, 0), (8, 2, 0), (8, 1, 0),
                                            (16, 2, 1), (32, 8, 1)])
def test_batched_decode_vs_oracle(H, Hk, rope_type):
    rng = np.random.default_rng(1280 + H + Hk + rope_type)
    ms, n_layers, layer = 400, 2, 1
    kv = Hk * HD
    lengths = [0, 1, 15, 16, 17, 63, 64, 65, 255, 399]
    n = len(lengths)
    tables = O.rope_tables(ms, HD, 10000.0)
    with pb.Attn(n_layers, H, Hk, ms, rope_type=rope_type, n_seqs=n, head_dim=HD) as at:
        caches = []
        for s in range(n):
            kc = random_cache(rng, ms, kv)
            vc = random_cache(rng, ms, kv)
            at.kv_upload(s, layer, 0, kc, vc)
            caches.append((kc, vc))
        q = rng.standard_normal((n, H * HD), dtype=np.float32) * 2
        k = rng.standard_normal((n, kv), dtype=np.float32) * 2
        v = rng.standard_normal((n, kv), dtype=np.float32)
        seqs = np.arange(n, dtype=np.int32)[::-1].copy()
        pos = np.array(lengths, np.int32)
        out = at.decode_batch(layer, seqs, pos, q, k, v)
        for i in range(n):
            s = int(seqs[i])
            kc, vc = caches[s]
            want, kc2, vc2 = oracle_decode_layer(H, Hk, ms, kc, vc, int(pos[i]), q[i], k[i],
                                                 v[i], tables, rope_type, hd=HD)
            gk, gv = at.kv_download(s, layer, 0, ms)
            np.testing.assert_array_equal(gk, kc2)
            np.testing.assert_array_equal(gv, vc2)
            assert_attn_close(out[i], want, f"hd128 H{H} Hk{Hk} seq {s} pos {pos[i]}")
        gk, _ = at.kv_download(0, 0, 0, ms)
        assert not gk.any()


def test_long_context_split():
    # LLaMA-3-8B-like heads (32/8, theta 5e5) over 8192 rows: many segments
    # and the merge kernel
    rng = np.random.default_rng(12)
    H, Hk, ms = 32, 8, 8192
    tables = O.rope_tables(ms, HD, 500000.0)
    kc = random_cache(rng, ms, Hk * HD)
    vc = random_cache(rng, ms, Hk * HD)
    q = rng.standard_normal(H * HD, dtype=np.float32)
    k = rng.standard_normal(Hk * HD, dtype=np.float32)
    v = rng.standard_normal(Hk * HD, dtype=np.float32)
    with pb.Attn(1, H, Hk, ms, rope_base=500000.0, head_dim=HD) as at:
        at.kv_upload(0, 0, 0, kc, vc)
        got = at.decode(0, 0, ms - 1, q, k, v)
    want, _, _ = oracle_decode_layer(H, Hk, ms, kc, vc, ms - 1, q, k, v, tables, hd=HD)
    assert_attn_close(got, want, "hd128 8192 rows")


@pytest.mark.parametrize("H,Hk,start,n_tok,rope_type", [
    (8, 2, 0, 1, 0), (8, 2, 0, 130, 0), (32, 8, 77, 200, 0), (16, 2, 5, 150, 1),
    (32, 4, 0, 1100, 0), (8, 8, 0, 300, 0), (8, 1, 3, 190, 0)])
def test_prefill_vs_oracle(H, Hk, start, n_tok, rope_type):
    rng = np.random.default_rng(2000 + H + Hk + start + n_tok)
    ms = start + n_tok + 16
    kv = Hk * HD
    tables = O.rope_tables(ms, HD, 10000.0)
    kc = np.zeros((ms, kv), np.uint16)
    vc = np.zeros((ms, kv), np.uint16)
    if start:
        kc[:start] = random_cache(rng, start, kv)
        vc[:start] = random_cache(rng, start, kv)
    q = rng.standard_normal((n_tok, H * HD), dtype=np.float32)
    k = rng.standard_normal((n_tok, kv), dtype=np.float32)
    v = rng.standard_normal((n_tok, kv), dtype=np.float32)
    with pb.Attn(1, H, Hk, ms, rope_type=rope_type, head_dim=HD) as at:
        at.kv_upload(0, 0, 0, kc, vc)
        got = at.prefill(0, 0, start, q, k, v)
        gk, gv = at.kv_download(0, 0, 0, ms)
    c = O.cfg(H, Hk, HD, ms, rope_type)
    kc2, vc2 = kc.copy(), vc.copy()
    want, _, _ = O.attn_prefill(c, kc2.ravel(), vc2.ravel(), start, q, k, v, *tables)
    np.testing.assert_array_equal(gk, kc2)
    np.testing.assert_array_equal(gv, vc2)
    assert_attn_close(got, want, f"hd128 prefill H{H} Hk{Hk} start{start} n{n_tok}")


def test_prefill_out_stride():
    rng = np.random.default_rng(3)
    H, Hk, ms, n = 8, 2, 256, 70
    q = rng.standard_normal((n, H * HD), dtype=np.float32)
    k = rng.standard_normal((n, Hk * HD), dtype=np.float32)
    v = rng.standard_normal((n, Hk * HD), dtype=np.float32)
    with pb.Attn(1, H, Hk, ms, head_dim=HD) as at:
        a = at.prefill(0, 0, 0, q, k, v)
    with pb.Attn(1, H, Hk, ms, head_dim=HD) as at:
        b = at.prefill(0, 0, 0, q, k, v, out_stride=H * HD + 96)
    np.testing.assert_array_equal(a, b[:, :H * HD])
    assert not b[:, H * HD:].any()


def test_rope_entry_bit_exact():
    # pl_attn_rope at head_dim 128, both pairings, against the oracle rotation
    rng = np.random.default_rng(5)
    H, Hk, ms, n = 8, 2, 64, 9
    for rope_type in (0, 1):
        ct, st = O.rope_tables(ms, HD, 10000.0)
        q = rng.standard_normal((n, H * HD), dtype=np.float32) * 3
        k = rng.standard_normal((n, Hk * HD), dtype=np.float32) * 3
        with pb.Attn(1, H, Hk, ms, rope_type=rope_type, head_dim=HD) as at:
            gq, gk = at.rope(20, q, k)
        for r in range(n):
            wq, wk = q[r].copy(), k[r].copy()
            p = 20 + r
            O.port().orc_rope(wq, wk, HD, H, Hk, np.ascontiguousarray(ct[p * 64:(p + 1) * 64]),
                              np.ascontiguousarray(st[p * 64:(p + 1) * 64]), rope_type)
            np.testing.assert_array_equal(gq[r].view(np.uint32), wq.view(np.uint32))
            np.testing.assert_array_equal(gk[r].view(np.uint32), wk.view(np.uint32))


def test_kv_split_partials_and_combine():
    # three shards of one sequence through pl_attn_decode_partial_dev and the
    # LSE merge of pl_attn_combine_dev equal the unsplit decode
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(13)
    H, Hk, P = 32, 8, 3000
    ms = P + 8
    kv = Hk * HD
    tables = O.rope_tables(ms, HD, 10000.0)
    kc = random_cache(rng, ms, kv)
    vc = random_cache(rng, ms, kv)
    q = rng.standard_normal(H * HD, dtype=np.float32)
    k = rng.standard_normal(kv, dtype=np.float32)
    v = rng.standard_normal(kv, dtype=np.float32)
    want, kc2, vc2 = oracle_decode_layer(H, Hk, ms, kc, vc, P, q, k, v, tables, hd=HD)
    bounds = [0, 1000, 2000, P + 1]
    dev = torch.device("cuda", 0)
    with pb.Attn(3, H, Hk, ms, head_dim=HD) as at:
        assert at.part_stride == HD + 4
        for g in range(3):   # shard g lives in layer g of the same slot
            lo, hi = bounds[g], bounds[g + 1]
            rows = min(hi, P) - lo
            at.kv_upload(0, g, 0, kc[lo:lo + rows], vc[lo:lo + rows])
        dq = torch.from_numpy(q).to(dev)
        dk = torch.from_numpy(k).to(dev)
        dv = torch.from_numpy(v).to(dev)
        parts = torch.empty(3, H * at.part_stride, device=dev)
        out = torch.empty(H * HD, device=dev)
        st = torch.cuda.current_stream(dev).cuda_stream
        for g in range(3):
            lo, hi = bounds[g], bounds[g + 1]
            at.decode_partial_dev(0, g, P, lo, hi - lo, g == 2, dq.data_ptr(), dk.data_ptr(),
                                  dv.data_ptr(), parts[g].data_ptr(), st)
        at.combine_dev(3, parts.data_ptr(), out.data_ptr(), st)
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        gk, gv = at.kv_download(0, 2, P - 2000, 1)
    np.testing.assert_array_equal(gk[0], kc2[P])
    np.testing.assert_array_equal(gv[0], vc2[P])
    assert_attn_close(got, want, "hd128 3-shard combine")


def test_no_alloc_entry_point():
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(14)
    H, Hk, ms, n = 32, 8, 300, 5
    kv = Hk * HD
    tables = O.rope_tables(ms, HD, 10000.0)
    dev = torch.device("cuda", 0)
    with pb.Attn(1, H, Hk, ms, n_seqs=n, head_dim=HD) as at:
        caches = []
        for s in range(n):
            kc, vc = random_cache(rng, ms, kv), random_cache(rng, ms, kv)
            at.kv_upload(s, 0, 0, kc, vc)
            caches.append((kc, vc))
        q = rng.standard_normal((n, H * HD), dtype=np.float32)
        k = rng.standard_normal((n, kv), dtype=np.float32)
        v = rng.standard_normal((n, kv), dtype=np.float32)
        pos = np.array([0, 5, 100, 256, 299], np.int32)
        seqs = np.arange(n, dtype=np.int32)
        t = {name: torch.from_numpy(x).to(dev) for name, x in
             dict(q=q, k=k, v=v, pos=pos, seqs=seqs).items()}
        out = torch.empty(n, H * HD, device=dev)
        at.decode_batch_dev_noalloc(0, n, t["seqs"].data_ptr(), t["pos"].data_ptr(), 299,
                                    t["q"].data_ptr(), t["k"].data_ptr(), t["v"].data_ptr(),
                                    out.data_ptr(), torch.cuda.current_stream(dev).cuda_stream)
        torch.cuda.synchronize()
        got = out.cpu().numpy()
    for i in range(n):
        kc, vc = caches[i]
        want, _, _ = oracle_decode_layer(H, Hk, ms, kc, vc, int(pos[i]), q[i], k[i], v[i],
                                         tables, hd=HD)
        assert_attn_close(got[i], want, f"hd128 noalloc seq {i}")
