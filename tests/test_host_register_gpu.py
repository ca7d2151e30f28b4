"""pl_attn_host_register: host-buffer calls whose inputs and outputs lie in
registered (page-locked, mapped) caller memory move them directly between
the caller and the device: q by one copy, k, v and the output by the
kernels over the bus.  Results must equal the staged path bit for bit; the error
cases return status codes and leave the module usable."""
import numpy as np
import pytest

import picolm_b200 as pb
from tests.util import random_cache

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _built():
    from picolm_b200 import build
    build.build()


def _inputs(rng, n, q_dim, kv_dim):
    return (rng.standard_normal((n, q_dim), dtype=np.float32),
            rng.standard_normal((n, kv_dim), dtype=np.float32),
            rng.standard_normal((n, kv_dim), dtype=np.float32))


def test_decode_batch_registered_equals_staged():
    rng = np.random.default_rng(31)
    H, Hk, ms, n = 32, 4, 300, 6
    pos = np.array([0, 3, 64, 127, 200, 299], np.int32)
    seqs = np.arange(n, dtype=np.int32)
    q, k, v = _inputs(rng, n, H * 64, Hk * 64)
    caches = [(random_cache(rng, ms, Hk * 64), random_cache(rng, ms, Hk * 64)) for _ in range(n)]
    results = []
    # registered buffers: q is copied to the device, k and v are read and
    # the output written by the kernels over the bus (mapped).  A registered
    # range whose start is not 16-byte aligned, or a k without its v, takes
    # the staged route for that buffer; a q copied straight from the caller
    # with k and v staged ("q only", "misaligned") needs both copies.
    for mode in ("staged", "registered", "out only", "misaligned", "k only", "q only"):
        with pb.Attn(1, H, Hk, ms, n_seqs=n) as at:
            for s, (kc, vc) in enumerate(caches):
                at.kv_upload(s, 0, 0, kc, vc)
            qq, kk, vv = q.copy(), k.copy(), v.copy()
            out_buf = np.zeros(n * H * 64 + 4, np.float32)
            out = out_buf[1:1 + n * H * 64] if mode == "misaligned" else out_buf[:n * H * 64]
            regs = {"registered": (qq, kk, vv, out_buf), "out only": (out_buf,),
                    "misaligned": (qq, kk, vv, out_buf), "k only": (kk, out_buf),
                    "q only": (qq,)}.get(mode, ())
            if mode == "misaligned":
                vv_buf = np.zeros(vv.size + 4, np.float32)
                vv_buf[1:1 + vv.size] = vv.ravel()
                vv = vv_buf[1:1 + vv.size]
                regs = regs + (vv_buf,)
            for a in regs:
                at.host_register(a)
            at.decode_batch(0, seqs, pos, qq, kk, vv, out=out)
            gk, gv = at.kv_download(3, 0, 0, ms)
            for a in regs:
                at.host_unregister(a)
            results.append((out.copy(), gk, gv))
    for got in results[1:]:
        np.testing.assert_array_equal(got[0].view(np.uint32), results[0][0].view(np.uint32))
        np.testing.assert_array_equal(got[1], results[0][1])
        np.testing.assert_array_equal(got[2], results[0][2])


def test_prefill_registered_equals_staged():
    rng = np.random.default_rng(32)
    H, Hk, ms, n = 32, 4, 400, 333
    q, k, v = _inputs(rng, n, H * 64, Hk * 64)
    outs = []
    for registered in (False, True):
        with pb.Attn(1, H, Hk, ms) as at:
            qq, kk, vv = q.copy(), k.copy(), v.copy()
            out = np.zeros((n, H * 64), np.float32)
            if registered:
                for a in (qq, kk, vv, out):
                    at.host_register(a)
            got = at.prefill(0, 0, 7, qq, kk, vv, out=out)
            outs.append(np.array(got))
    np.testing.assert_array_equal(outs[1].view(np.uint32), outs[0].view(np.uint32))


def test_register_errors_leave_module_usable():
    rng = np.random.default_rng(33)
    H, Hk, ms = 8, 2, 64
    buf = np.zeros(1 << 16, np.float32)
    with pb.Attn(1, H, Hk, ms) as at:
        at.host_register(buf)
        # a range overlapping a registered one, and an address that starts none
        assert at.lib.pl_attn_host_register(buf.ctypes.data + 64, 1024) == pb.PL_EARG
        assert at.lib.pl_attn_host_unregister(buf.ctypes.data + 4) == pb.PL_EARG
        at.host_unregister(buf)
        assert at.lib.pl_attn_host_unregister(buf.ctypes.data) == pb.PL_EARG
        q, k, v = _inputs(rng, 1, H * 64, Hk * 64)
        out = at.decode(0, 0, 0, q[0], k[0], v[0])
        assert np.isfinite(out).all()


def test_single_sequence_decode_paths():
    """One sequence per call: up to 8 tiles one CTA reads q, k and v over the
    bus, from registered buffers or the mapped staging area, and no copy is
    queued; past that q, k and v go to the device in one copy and the split
    merge follows.  Every path against the oracle, registered equal to
    staged bit for bit, and the appended row bit-exact."""
    from oracle import oracle as O
    from tests.util import assert_attn_close
    rng = np.random.default_rng(34)
    H, Hk, ms = 32, 4, 700
    kv = Hk * 64
    kc = random_cache(rng, ms, kv)
    vc = random_cache(rng, ms, kv)
    tables = O.rope_tables(ms, 64, 10000.0)
    c = O.cfg(H, Hk, 64, ms)
    for p in (0, 100, 255, 256, 600):
        q, k, v = (x[0] for x in _inputs(rng, 1, H * 64, kv))
        fk, fv = kc.copy(), vc.copy()
        want, _, _ = O.attn_decode(c, fk.ravel(), fv.ravel(), p, q, k, v, *tables)
        outs = []
        for registered in (False, True):
            with pb.Attn(1, H, Hk, ms) as at:
                if p:
                    at.kv_upload(0, 0, 0, kc[:p], vc[:p])
                qq, kk, vv = q.copy(), k.copy(), v.copy()
                out = np.zeros(H * 64, np.float32)
                regs = (qq, kk, vv, out) if registered else ()
                for a in regs:
                    at.host_register(a)
                at.decode_batch(0, [0], [p], qq, kk, vv, out=out)
                gk, gv = at.kv_download(0, 0, p, 1)
                for a in regs:
                    at.host_unregister(a)
            np.testing.assert_array_equal(np.ravel(gk), fk[p])
            np.testing.assert_array_equal(np.ravel(gv), fv[p])
            assert_attn_close(out, want, f"decode at {p}, registered={registered}")
            outs.append(out.copy())
        np.testing.assert_array_equal(outs[1].view(np.uint32), outs[0].view(np.uint32))


@pytest.mark.parametrize("n", [128, 129])
def test_decode_batch_inline_boundary(n):
    """Up to 128 sequences carry their slots and positions in the kernel
    arguments; 129 stage them and copy them after the gathered q.  Both,
    with registered and staged buffers, against each other bit for bit and
    against the oracle on a sample of sequences."""
    from oracle import oracle as O
    from tests.util import assert_attn_close
    rng = np.random.default_rng(35 + n)
    H, Hk, ms = 32, 4, 96
    kv = Hk * 64
    pos = rng.integers(0, ms, n).astype(np.int32)
    seqs = rng.permutation(n).astype(np.int32)
    q, k, v = _inputs(rng, n, H * 64, kv)
    caches = [(random_cache(rng, ms, kv), random_cache(rng, ms, kv)) for _ in range(n)]
    outs = []
    for registered in (False, True):
        with pb.Attn(1, H, Hk, ms, n_seqs=n) as at:
            for s, (kc, vc) in enumerate(caches):
                at.kv_upload(s, 0, 0, kc, vc)
            qq, kk, vv = q.copy(), k.copy(), v.copy()
            out = np.zeros(n * H * 64, np.float32)
            regs = (qq, kk, vv, out) if registered else ()
            for a in regs:
                at.host_register(a)
            at.decode_batch(0, seqs, pos, qq, kk, vv, out=out)
            for a in regs:
                at.host_unregister(a)
            outs.append(out.reshape(n, H * 64).copy())
    np.testing.assert_array_equal(outs[1].view(np.uint32), outs[0].view(np.uint32))
    tables = O.rope_tables(ms, 64, 10000.0)
    c = O.cfg(H, Hk, 64, ms)
    for i in (0, 1, n // 2, n - 1):
        kc, vc = (x.copy() for x in caches[seqs[i]])
        want, _, _ = O.attn_decode(c, kc.ravel(), vc.ravel(), int(pos[i]), q[i], k[i], v[i],
                                   *tables)
        assert_attn_close(outs[1][i], want, f"n={n} sequence {i}")


def test_decode_batch_registered_hd128_qwen():
    """head_dim 128 and Qwen pairing through the host-buffer decode: q
    gathered over the bus (16 KB a sequence), k and v read and the output
    written over the bus from registered buffers; against the staged call
    bit for bit and against the oracle."""
    from oracle import oracle as O
    from tests.util import assert_attn_close
    rng = np.random.default_rng(36)
    H, Hk, hd, ms, n = 32, 8, 128, 160, 12
    kv = Hk * hd
    pos = rng.integers(0, ms, n).astype(np.int32)
    seqs = np.arange(n, dtype=np.int32)
    q, k, v = _inputs(rng, n, H * hd, kv)
    caches = [(random_cache(rng, ms, kv), random_cache(rng, ms, kv)) for _ in range(n)]
    outs = []
    for registered in (False, True):
        with pb.Attn(1, H, Hk, ms, n_seqs=n, head_dim=hd, rope_type=1,
                     rope_base=1000000.0) as at:
            for s, (kc, vc) in enumerate(caches):
                at.kv_upload(s, 0, 0, kc, vc)
            qq, kk, vv = q.copy(), k.copy(), v.copy()
            out = np.zeros(n * H * hd, np.float32)
            regs = (qq, kk, vv, out) if registered else ()
            for a in regs:
                at.host_register(a)
            at.decode_batch(0, seqs, pos, qq, kk, vv, out=out)
            for a in regs:
                at.host_unregister(a)
            outs.append(out.reshape(n, H * hd).copy())
    np.testing.assert_array_equal(outs[1].view(np.uint32), outs[0].view(np.uint32))
    tables = O.rope_tables(ms, hd, 1000000.0)
    c = O.cfg(H, Hk, hd, ms, 1)
    for i in range(n):
        kc, vc = (x.copy() for x in caches[i])
        want, _, _ = O.attn_decode(c, kc.ravel(), vc.ravel(), int(pos[i]), q[i], k[i], v[i],
                                   *tables)
        assert_attn_close(outs[1][i], want, f"hd128 qwen sequence {i}")
