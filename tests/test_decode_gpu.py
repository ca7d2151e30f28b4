"""Decode parity: the CUDA path (through the C ABI) against the oracle.

KV rows must be bit-identical to picolm's (FP16 append with ties-away
rounding, unfused RoPE); attention outputs within max-abs 2e-3 / rel 1e-2.
"""
import numpy as np
import pytest

import picolm_b200 as pb
from oracle import oracle as O
from tests.util import assert_attn_close, oracle_decode_layer, random_cache

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _built():
    from picolm_b200 import build
    build.build()


@pytest.mark.parametrize("pos", [0, 1, 17, 63])
def test_golden_small_gqa(golden, pos):
    # model_forward_ex of the genuine reference, H=8, Hk=2, max_seq=64
    with pb.Attn(1, 8, 2, 64) as at:
        at.kv_upload(0, 0, 0, golden["dsm_kc0"], golden["dsm_vc0"])
        out = at.decode(0, 0, int(pos), golden[f"dsm_p{pos}_q"], golden[f"dsm_p{pos}_k"],
                        golden[f"dsm_p{pos}_v"])
        kc, vc = at.kv_download(0, 0, 0, 64)
    np.testing.assert_array_equal(kc[pos], golden[f"dsm_p{pos}_krow"])
    np.testing.assert_array_equal(vc[pos], golden[f"dsm_p{pos}_vrow"])
    mask = np.arange(64) != pos
    np.testing.assert_array_equal(kc[mask], golden["dsm_kc0"][mask])
    assert_attn_close(out, golden[f"dsm_p{pos}_out"], f"golden pos {pos}")


def test_golden_config1(golden):
    from tests.test_oracle import config1_inputs
    _, _, _, _, kc0, vc0 = config1_inputs()
    with pb.Attn(1, 32, 4, 256) as at:
        at.kv_upload(0, 0, 0, kc0, vc0)
        out = at.decode(0, 0, 255, golden["c1_q"], golden["c1_k"], golden["c1_v"])
        kc, vc = at.kv_download(0, 0, 255, 1)
    np.testing.assert_array_equal(kc[0], golden["c1_krow"])
    np.testing.assert_array_equal(vc[0], golden["c1_vrow"])
    assert_attn_close(out, golden["c1_out"], "config 1")


@pytest.mark.parametrize("H,Hk,rope_type", [(32, 4, 0), (32, 8, 0), (8, 1, 0), (8, 8, 0),
                                            (16, 2, 1), (32, 4, 1)])
def test_batched_decode_vs_oracle(H, Hk, rope_type):
    rng = np.random.default_rng(100 + H + Hk + rope_type)
    ms, n_layers, layer = 600, 2, 1
    kv = Hk * 64
    lengths = [0, 1, 15, 16, 31, 32, 33, 127, 128, 129, 255, 599]
    n = len(lengths)
    tables = O.rope_tables(ms, 64, 10000.0)
    with pb.Attn(n_layers, H, Hk, ms, rope_type=rope_type, n_seqs=n) as at:
        caches = []
        for s in range(n):
            kc = random_cache(rng, ms, kv)
            vc = random_cache(rng, ms, kv)
            at.kv_upload(s, layer, 0, kc, vc)
            caches.append((kc, vc))
        q = rng.standard_normal((n, H * 64), dtype=np.float32) * 2
        k = rng.standard_normal((n, kv), dtype=np.float32) * 2
        v = rng.standard_normal((n, kv), dtype=np.float32)
        seqs = np.arange(n, dtype=np.int32)[::-1].copy()   # slot order != batch order
        pos = np.array(lengths, np.int32)
        out = at.decode_batch(layer, seqs, pos, q, k, v)
        for i in range(n):
            s = int(seqs[i])
            kc, vc = caches[s]
            want, kc2, vc2 = oracle_decode_layer(H, Hk, ms, kc, vc, int(pos[i]), q[i], k[i],
                                                 v[i], tables, rope_type)
            gk, gv = at.kv_download(s, layer, 0, ms)
            np.testing.assert_array_equal(gk, kc2)
            np.testing.assert_array_equal(gv, vc2)
            assert_attn_close(out[i], want, f"seq {s} pos {pos[i]}")
        # the other layer is untouched
        gk, _ = at.kv_download(0, 0, 0, ms)
        assert not gk.any()


def test_decode_sequence_of_steps():
    # 70 consecutive decode steps from an empty cache, as picolm's generation
    # loop runs them (picolm.c:251-275): every step appends and attends.
    rng = np.random.default_rng(7)
    H, Hk, ms = 32, 4, 96
    tables = O.rope_tables(ms, 64, 10000.0)
    kc = np.zeros((ms, Hk * 64), np.uint16)
    vc = np.zeros((ms, Hk * 64), np.uint16)
    with pb.Attn(1, H, Hk, ms) as at:
        for p in range(70):
            q = rng.standard_normal(H * 64, dtype=np.float32)
            k = rng.standard_normal(Hk * 64, dtype=np.float32)
            v = rng.standard_normal(Hk * 64, dtype=np.float32)
            got = at.decode(0, 0, p, q, k, v)
            want, kc, vc = oracle_decode_layer(H, Hk, ms, kc, vc, p, q, k, v, tables)
            assert_attn_close(got, want, f"step {p}")
        gk, gv = at.kv_download(0, 0, 0, ms)
    np.testing.assert_array_equal(gk, kc)
    np.testing.assert_array_equal(gv, vc)


def test_long_context_split():
    # long enough that the KV split uses many CTAs and the combine kernel
    rng = np.random.default_rng(9)
    H, Hk, ms = 32, 8, 8192
    tables = O.rope_tables(ms, 64, 500000.0)
    kc = random_cache(rng, ms, Hk * 64)
    vc = random_cache(rng, ms, Hk * 64)
    q = rng.standard_normal(H * 64, dtype=np.float32)
    k = rng.standard_normal(Hk * 64, dtype=np.float32)
    v = rng.standard_normal(Hk * 64, dtype=np.float32)
    with pb.Attn(1, H, Hk, ms, rope_base=500000.0) as at:
        at.kv_upload(0, 0, 0, kc, vc)
        got = at.decode(0, 0, ms - 1, q, k, v)
    want, _, _ = oracle_decode_layer(H, Hk, ms, kc, vc, ms - 1, q, k, v, tables)
    assert_attn_close(got, want, "8192 rows")


def test_rope_bit_exact():
    rng = np.random.default_rng(3)
    H, Hk, ms = 32, 4, 512
    for rope_type in (0, 1):
        tables = O.rope_tables(ms, 64, 10000.0)
        q = rng.standard_normal((5, H * 64), dtype=np.float32) * 10
        k = rng.standard_normal((5, Hk * 64), dtype=np.float32) * 10
        with pb.Attn(1, H, Hk, ms, rope_type=rope_type) as at:
            gq, gk = at.rope(300, q, k)
        half = 32
        for r in range(5):
            wq, wk = q[r].copy(), k[r].copy()
            O.port().orc_rope(wq, wk, 64, H, Hk,
                              np.ascontiguousarray(tables[0][(300 + r) * half:(301 + r) * half]),
                              np.ascontiguousarray(tables[1][(300 + r) * half:(301 + r) * half]),
                              rope_type)
            np.testing.assert_array_equal(gq[r].view(np.uint32), wq.view(np.uint32))
            np.testing.assert_array_equal(gk[r].view(np.uint32), wk.view(np.uint32))


def test_set_rope_tables_from_host():
    # a caller's own tables (model.c's s->rope_cos/sin) replace the module's
    rng = np.random.default_rng(4)
    H, Hk, ms = 8, 2, 32
    c = rng.uniform(-1, 1, ms * 32).astype(np.float32)
    s = rng.uniform(-1, 1, ms * 32).astype(np.float32)
    q = rng.standard_normal(H * 64, dtype=np.float32)
    with pb.Attn(1, H, Hk, ms) as at:
        at.set_rope(c, s)
        gq, _ = at.rope(5, q, None)
    wq = q.copy()
    O.port().orc_rope(wq, np.zeros(Hk * 64, np.float32), 64, H, Hk,
                      np.ascontiguousarray(c[5 * 32:6 * 32]),
                      np.ascontiguousarray(s[5 * 32:6 * 32]), 0)
    np.testing.assert_array_equal(gq.view(np.uint32), wq.view(np.uint32))


def test_kv_roundtrip_and_argument_errors():
    rng = np.random.default_rng(5)
    with pb.Attn(3, 32, 4, 128, n_seqs=2) as at:
        k = random_cache(rng, 40, 256)
        v = random_cache(rng, 40, 256)
        at.kv_upload(1, 2, 50, k, v)
        gk, gv = at.kv_download(1, 2, 50, 40)
        np.testing.assert_array_equal(gk, k)
        np.testing.assert_array_equal(gv, v)
        q = np.zeros(2048, np.float32)
        kk = np.zeros(256, np.float32)
        for args in [(2, 0, 0), (0, 3, 0), (0, 0, 128), (-1, 0, 0), (0, 0, -1)]:
            with pytest.raises(pb.PlAttnError) as ei:
                at.decode(*args, q, kk, kk)
            assert ei.value.rc == pb.PL_EARG
        with pytest.raises(pb.PlAttnError):
            at.decode_batch(0, [0, 0], [1, 2], np.zeros((2, 2048)), np.zeros((2, 256)),
                            np.zeros((2, 256)))
        with pytest.raises(pb.PlAttnError):
            at.kv_download(0, 0, 100, 40)
        # a second init while one is live is refused
        assert at.lib.pl_attn_init(1, 32, 4, 64, 64, 1e4, 0, 1, 0) == pb.PL_ESTATE
        # the context is still usable after the refusals
        out = at.decode(0, 0, 0, q, kk, kk)
        assert np.all(np.isfinite(out))


def test_kv_split_partials_and_combine():
    # one long sequence whose rows live in three shards (three slots on one
    # device here; three devices in the multi-GPU path).  Shard partials
    # merged by the LSE combine equal the unsplit decode.
    import torch
    rng = np.random.default_rng(11)
    H, Hk, ms = 32, 8, 1024
    P = 1000                       # the new token's position
    bounds = [0, 333, 700, P + 1]  # shard g holds global rows [b_g, b_{g+1})
    tables = O.rope_tables(ms, 64, 500000.0)
    kc = random_cache(rng, ms, Hk * 64)
    vc = random_cache(rng, ms, Hk * 64)
    q = rng.standard_normal(H * 64, dtype=np.float32)
    k = rng.standard_normal(Hk * 64, dtype=np.float32)
    v = rng.standard_normal(Hk * 64, dtype=np.float32)
    want, kc2, _ = oracle_decode_layer(H, Hk, ms, kc, vc, P, q, k, v, tables)
    dev = torch.device("cuda:0")
    with pb.Attn(1, H, Hk, ms, rope_base=500000.0, n_seqs=3) as at:
        for g in range(3):
            lo, hi = bounds[g], bounds[g + 1]
            at.kv_upload(g, 0, 0, kc[lo:hi], vc[lo:hi])
        dq = torch.from_numpy(q).to(dev)
        dk = torch.from_numpy(k).to(dev)
        dv = torch.from_numpy(v).to(dev)
        parts = torch.empty(3, H * pb.PART_STRIDE, device=dev)
        out = torch.empty(H * 64, device=dev)
        st = torch.cuda.current_stream().cuda_stream
        for g in range(3):
            lo, hi = bounds[g], bounds[g + 1]
            at.decode_partial_dev(g, 0, P, lo, hi - lo, g == 2, dq.data_ptr(), dk.data_ptr(),
                                  dv.data_ptr(), parts[g].data_ptr(), st)
        at.combine_dev(3, parts.data_ptr(), out.data_ptr(), st)
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        rk, _ = at.kv_download(2, 0, P - bounds[2], 1)
    np.testing.assert_array_equal(rk[0], kc2[P])
    assert_attn_close(got, want, "3-shard combine")


def test_batch_over_one_launch():
    # 1100 sequences: more than one launch holds (1024), so the call runs the
    # decode kernel and merge twice; sequences on both sides of the chunk
    # edge, and the first and last, against the oracle
    rng = np.random.default_rng(41)
    H, Hk, ms, n = 8, 2, 48, 1100
    kv = Hk * 64
    tables = O.rope_tables(ms, 64, 10000.0)
    pos = rng.integers(0, ms, n).astype(np.int32)
    pos[[0, 1023, 1024, n - 1]] = [ms - 1, 0, ms - 1, 17]
    seqs = rng.permutation(n).astype(np.int32)
    q = rng.standard_normal((n, H * 64), dtype=np.float32)
    k = rng.standard_normal((n, kv), dtype=np.float32)
    v = rng.standard_normal((n, kv), dtype=np.float32)
    check = [0, 1, 500, 1022, 1023, 1024, 1025, n - 1]
    with pb.Attn(1, H, Hk, ms, n_seqs=n) as at:
        caches = {}
        for i in check:
            s = int(seqs[i])
            caches[s] = (random_cache(rng, ms, kv), random_cache(rng, ms, kv))
            at.kv_upload(s, 0, 0, *caches[s])
        out = at.decode_batch(0, seqs, pos, q, k, v).reshape(n, H * 64)
        for i in check:
            s = int(seqs[i])
            kc, vc = caches[s]
            want, kc2, vc2 = oracle_decode_layer(H, Hk, ms, kc, vc, int(pos[i]), q[i], k[i], v[i],
                                                 tables)
            gk, gv = at.kv_download(s, 0, 0, ms)
            np.testing.assert_array_equal(gk, kc2)
            np.testing.assert_array_equal(gv, vc2)
            assert_attn_close(out[i], want, f"batch of {n}: entry {i} (slot {s}, pos {pos[i]})")


def test_dev_steps_with_positions_written_just_before():
    # Device-pointer decode steps queued back to back with no host
    # synchronisation, as an engine drives them.  Before each step a kernel on
    # the same stream writes that step's slots and positions into the SAME two
    # arrays, right before the decode launch.  The decode grid is launched
    # with programmatic stream serialisation and may start its set-up while
    # the kernel before it finishes; what it reads then is only a hint, checked
    # after griddepcontrol.wait.  The batch order of the slots changes every
    # step, so a stale hint would partition the tiles differently.  Every
    # step's output and the final caches against the oracle.
    import torch
    rng = np.random.default_rng(53)
    H, Hk, ms, n, steps = 32, 4, 320, 24, 6
    kv = Hk * 64
    tables = O.rope_tables(ms, 64, 10000.0)
    base = rng.integers(1, ms - steps, n).astype(np.int32)
    base[[0, 1]] = [ms - steps, 0]          # the longest cache and an empty one
    order = np.stack([rng.permutation(n) for _ in range(steps)]).astype(np.int32)
    pos_all = np.stack([base[order[s]] + s for s in range(steps)]).astype(np.int32)
    q = rng.standard_normal((steps, n, H * 64), dtype=np.float32)
    k = rng.standard_normal((steps, n, kv), dtype=np.float32)
    v = rng.standard_normal((steps, n, kv), dtype=np.float32)
    caches = []
    for s in range(n):
        kc = np.zeros((ms, kv), np.uint16)
        vc = np.zeros((ms, kv), np.uint16)
        kc[:base[s]] = random_cache(rng, int(base[s]), kv)
        vc[:base[s]] = random_cache(rng, int(base[s]), kv)
        caches.append((kc, vc))
    dev = torch.device("cuda", 0)
    with pb.Attn(1, H, Hk, ms, n_seqs=n) as at:
        for s in range(n):
            at.kv_upload(s, 0, 0, *caches[s])
        d_order = torch.from_numpy(order).to(dev)
        d_pos_all = torch.from_numpy(pos_all).to(dev)
        dq, dk, dv = (torch.from_numpy(x).to(dev) for x in (q, k, v))
        d_seqs = torch.full((n,), -1, dtype=torch.int32, device=dev)
        d_pos = torch.full((n,), -1, dtype=torch.int32, device=dev)
        out = torch.full((steps, n, H * 64), float("nan"), device=dev)
        zero = torch.zeros((), dtype=torch.int32, device=dev)
        st = torch.cuda.current_stream().cuda_stream
        torch.cuda.synchronize()
        for s in range(steps):
            torch.add(d_order[s], zero, out=d_seqs)    # elementwise kernels, not copies
            torch.add(d_pos_all[s], zero, out=d_pos)
            at.decode_batch_dev(0, n, d_seqs.data_ptr(), d_pos.data_ptr(), ms - 1,
                                dq[s].data_ptr(), dk[s].data_ptr(), dv[s].data_ptr(),
                                out[s].data_ptr(), st)
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        for s in range(steps):
            for i in range(n):
                slot = int(order[s, i])
                kc, vc = caches[slot]
                want, kc, vc = oracle_decode_layer(H, Hk, ms, kc, vc, int(pos_all[s, i]),
                                                   q[s, i], k[s, i], v[s, i], tables)
                caches[slot] = (kc, vc)
                assert_attn_close(got[s, i], want, f"step {s} entry {i} (slot {slot})")
        for slot in range(n):
            gk, gv = at.kv_download(slot, 0, 0, ms)
            np.testing.assert_array_equal(gk, caches[slot][0])
            np.testing.assert_array_equal(gv, caches[slot][1])
