"""Failure paths, made on the host or by a wait that nothing releases (GPU).

* A KV-split merge whose peer never arrives: two processes on one GPU map
  each other's receive buffers (pl_attn_xfer_setup / _connect); rank 1 stays
  alive but never calls pl_attn_combine_p2p_dev (or pl_attn_decode_p2p_dev,
  where every block of the merge grid waits for its head).  Rank 0's merge
  kernel stores its partial (each value beside the merge's epoch) and
  waits, bounded by the limit set with pl_attn_set_wait_limit (50 ms here),
  for rank 1's values to show that epoch, which never happens.
  pl_attn_status must report PL_ETIMEOUT, and the module must stay usable: a
  decode right after matches the oracle.  Only one kernel waits, on values
  no one writes, so nothing depends on two kernels running at once;
  rank 1 leaves only after rank 0 has finished, so no mapping disappears
  under a running kernel.  This is the failure picolm's Vulkan backend
  detects with its 5 s fence timeout (picolm/gpu.c:693-698).
* Allocation failures: PL_ATTN_FAIL_ALLOC=n makes the module's n-th
  allocation after pl_attn_init fail as an exhausted device would.  For
  every n that lands in init or in a later call's lazy allocation, the
  call reports PL_ENOMEM, leaves the module consistent, and the same call
  retried succeeds with the oracle's result.
"""
import multiprocessing as mp
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


def _silent_rank(conn):
    """Rank 1: sets up and connects, then waits until rank 0 is done."""
    import picolm_b200 as pb
    with pb.Attn(1, 8, 2, 64) as at:
        conn.send(at.xfer_setup(2, 1))
        handles = conn.recv()
        at.xfer_connect(handles)
        conn.send("connected")
        conn.recv()  # "done": rank 0 has finished every kernel that touches our buffer
    conn.send("closed")


@pytest.mark.parametrize("fused", [False, True], ids=["combine_p2p", "decode_p2p"])
def test_p2p_merge_times_out_when_a_rank_never_arrives(fused):
    import torch
    ctx = mp.get_context("spawn")
    parent, child = ctx.Pipe()
    proc = ctx.Process(target=_silent_rank, args=(child,), daemon=True)
    proc.start()
    try:
        with pb.Attn(1, 8, 2, 64) as at:
            h0 = at.xfer_setup(2, 0)
            assert parent.poll(120), "rank 1 did not start"
            h1 = parent.recv()
            handles = [h0, h1]
            parent.send(handles)
            at.xfer_connect(handles)
            assert parent.poll(60) and parent.recv() == "connected"
            at.set_wait_limit(0.05)
            part = torch.zeros(8 * at.part_stride, device="cuda")
            out = torch.zeros(8 * 64, device="cuda")
            st = torch.cuda.current_stream().cuda_stream
            if fused:
                # partial over 11 (zero) cache rows, pushed, then the wait
                qd = torch.randn(8 * 64, device="cuda")
                at.decode_p2p_dev(0, 0, 10, 0, 11, 0, qd.data_ptr(), qd.data_ptr(),
                                  qd.data_ptr(), out.data_ptr(), st)
            else:
                at.combine_p2p_dev(part.data_ptr(), out.data_ptr(), st)
            assert at.status(st) == pb.PL_ETIMEOUT
            assert at.status(st) == pb.PL_OK  # the word was cleared
            at.set_wait_limit(2.0)
            # still usable: a decode against the oracle
            rng = np.random.default_rng(5)
            kc = random_cache(rng, 64, 128)
            vc = random_cache(rng, 64, 128)
            at.kv_upload(0, 0, 0, kc, vc)
            q = rng.standard_normal(8 * 64, dtype=np.float32)
            k = rng.standard_normal(128, dtype=np.float32)
            v = rng.standard_normal(128, dtype=np.float32)
            got = at.decode(0, 0, 40, q, k, v)
            want, _, _ = O.attn_decode(O.cfg(8, 2, 64, 64), kc.ravel(), vc.ravel(), 40, q, k, v,
                                       *O.rope_tables(64, 64, 10000.0))
            assert_attn_close(got, want, "decode after a timed-out merge")
        parent.send("done")
        assert parent.poll(60) and parent.recv() == "closed"
    finally:
        proc.join(60)
        if proc.is_alive():
            proc.kill()
    assert proc.exitcode == 0


def _run_calls(at, rng, state):
    """A host decode (staging + split partials) and a prefill (q16 staging):
    the lazy allocations after init.  Each call is retried once after
    PL_ENOMEM; returns how many calls failed that way."""
    H, Hk, ms = 8, 2, 600
    kv = Hk * 64
    tables = O.rope_tables(ms, 64, 10000.0)
    c = O.cfg(H, Hk, 64, ms)
    failures = 0

    def attempt(fn):
        nonlocal failures
        try:
            return fn()
        except pb.PlAttnError as e:
            assert e.rc == pb.PL_ENOMEM, e
            failures += 1
            return fn()  # the injected failure fires once

    kc, vc = state
    attempt(lambda: at.kv_upload(0, 0, 0, kc[:500], vc[:500]))
    q = rng.standard_normal(H * 64, dtype=np.float32)
    k = rng.standard_normal(kv, dtype=np.float32)
    v = rng.standard_normal(kv, dtype=np.float32)
    got = attempt(lambda: at.decode(0, 0, 500, q, k, v))
    want, _, _ = O.attn_decode(c, kc.ravel(), vc.ravel(), 500, q, k, v, *tables)
    assert_attn_close(got, want, "decode")
    qp = rng.standard_normal((40, H * 64), dtype=np.float32)
    kp = rng.standard_normal((40, kv), dtype=np.float32)
    vp = rng.standard_normal((40, kv), dtype=np.float32)
    gotp = attempt(lambda: at.prefill(0, 0, 501, qp, kp, vp))
    wantp, _, _ = O.attn_prefill(c, kc.ravel(), vc.ravel(), 501, qp, kp, vp, *tables)
    assert_attn_close(gotp, wantp, "prefill")
    return failures


def test_allocation_failures_report_enomem_and_recover(monkeypatch):
    rng0 = np.random.default_rng(6)
    kc0 = np.zeros((600, 128), np.uint16)
    vc0 = np.zeros((600, 128), np.uint16)
    kc0[:500] = random_cache(rng0, 500, 128)
    vc0[:500] = random_cache(rng0, 500, 128)
    in_init = in_calls = 0
    for n in range(1, 16):
        monkeypatch.setenv("PL_ATTN_FAIL_ALLOC", str(n))
        try:
            at = pb.Attn(1, 8, 2, 600)
        except pb.PlAttnError as e:
            assert e.rc == pb.PL_ENOMEM, e
            assert pb.load().pl_attn_available() == 0
            in_init += 1
            continue
        finally:
            monkeypatch.delenv("PL_ATTN_FAIL_ALLOC")
        with at:
            in_calls += _run_calls(at, np.random.default_rng(7), (kc0.copy(), vc0.copy()))
    assert in_init >= 5, in_init    # every allocation of init was hit once
    assert in_calls >= 3, in_calls  # staging, split partials, prefill q16
    # and a clean context afterwards
    with pb.Attn(1, 8, 2, 600) as at:
        assert _run_calls(at, np.random.default_rng(7), (kc0.copy(), vc0.copy())) == 0
