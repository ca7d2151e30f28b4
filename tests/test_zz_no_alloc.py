"""pl_attn_decode_batch_dev_noalloc against pl_attn_decode_batch_dev (GPU).

The no-allocation entry point exists for callers that cannot let the
library allocate device memory (engines that own the whole device through
their own pool; decode loops that cannot afford the device-wide
synchronisation a cudaMalloc/cudaFree may cause).  It must give the same
attention output as the ordinary device-pointer entry point, within the
suite's tolerance, on consecutive calls that share its static scratch.

This file is collected last on purpose, so that a run stopping at the first
failure has run every other test first.  Each test opens its own module
context, so the file passes alone in a fresh process or after the others.
"""
import os

import numpy as np
import pytest

import picolm_b200 as pb
from oracle import oracle as O
from tests.util import assert_attn_close, random_cache

pytestmark = pytest.mark.gpu


SCRATCH_PART_BYTES = 4 << 20  # the partial-slot part of the static array
N_SMS = 148                    # B200; every decode grid has at least one CTA per SM


def _setup(at, rng, n, ms, kv, lengths, caches=None):
    import torch
    dev = torch.device("cuda", 0)
    for s in range(n):
        kc, vc = random_cache(rng, ms, kv), random_cache(rng, ms, kv)
        at.kv_upload(s, 0, 0, kc, vc)
        if caches is not None:
            caches.append((kc, vc))
    q = torch.from_numpy(rng.standard_normal((n, at.q_dim), dtype=np.float32)).to(dev)
    k = torch.from_numpy(rng.standard_normal((n, kv), dtype=np.float32)).to(dev)
    v = torch.from_numpy(rng.standard_normal((n, kv), dtype=np.float32)).to(dev)
    seqs = torch.arange(n, dtype=torch.int32, device=dev)
    pos = torch.tensor(lengths, dtype=torch.int32, device=dev)
    return q, k, v, seqs, pos


@pytest.mark.parametrize("H,Hk,n,ms", [(32, 4, 64, 700), (32, 8, 1, 12000), (8, 2, 5, 90)])
def test_noalloc_matches_decode_batch_dev(H, Hk, n, ms):
    import torch
    rng = np.random.default_rng(77 + n)
    kv = Hk * 64
    lengths = [int(x) for x in rng.integers(0, ms, n)]
    lengths[0] = ms - 1
    with pb.Attn(1, H, Hk, ms, n_seqs=n) as at:
        q, k, v, seqs, pos = _setup(at, rng, n, ms, kv, lengths)
        st = torch.cuda.current_stream().cuda_stream
        want = torch.empty(n, H * 64, device="cuda")
        at.decode_batch_dev(0, n, seqs.data_ptr(), pos.data_ptr(), max(lengths), q.data_ptr(),
                            k.data_ptr(), v.data_ptr(), want.data_ptr(), st)
        # two calls in a row through the shared static scratch; each re-appends
        # the same K/V row, so the expected output does not change
        for call in range(2):
            got = torch.full((n, H * 64), float("nan"), device="cuda")
            at.decode_batch_dev_noalloc(0, n, seqs.data_ptr(), pos.data_ptr(), max(lengths),
                                        q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                        got.data_ptr(), st)
            torch.cuda.synchronize()
            assert_attn_close(got.cpu().numpy(), want.cpu().numpy(), f"call {call}")


def test_noalloc_rejects_too_many_sequences():
    import torch
    with pb.Attn(1, 8, 2, 64, n_seqs=1100) as at:
        d = torch.zeros(1100 * 512, device="cuda")
        idx = torch.zeros(1100, dtype=torch.int32, device="cuda")
        with pytest.raises(pb.PlAttnError) as ei:
            at.decode_batch_dev_noalloc(0, 1100, idx.data_ptr(), idx.data_ptr(), 0, d.data_ptr(),
                                        d.data_ptr(), d.data_ptr(), d.data_ptr())
        assert ei.value.rc == pb.PL_EARG


def test_noalloc_capped_grid_vs_oracle():
    """head_dim 128, 32 query heads over 8 KV heads, 200 sequences: a partial
    slot is 32 * 132 * 4 = 16896 bytes, so the 4 MiB hold 248 slots and only
    48 are left for CTAs after one per sequence.  The ordinary grid (at least
    one CTA per SM, at most one per tile) is larger, so this call runs the
    capped partition, fewer and longer CTAs, and is checked against the oracle
    as well as against the allocating entry point."""
    import torch
    H, Hk, hd, n, ms = 32, 8, 128, 200, 400
    kv = Hk * hd
    slots = SCRATCH_PART_BYTES // (H * (hd + 4) * 4)
    fit = slots - n
    rng = np.random.default_rng(91)
    lengths = [int(x) for x in rng.integers(64, ms - 1, n)]
    lengths[0] = ms - 1
    tp = 16  # tile rows at 8 KV heads x 128 (16 KB floor of 16 rows)
    tiles = sum((p + 1 + tp - 1) // tp for p in lengths)
    assert 1 <= fit < min(N_SMS, tiles), (fit, tiles)  # the cap applies
    caches = []
    with pb.Attn(1, H, Hk, ms, n_seqs=n, head_dim=hd, rope_base=500000.0) as at:
        q, k, v, seqs, pos = _setup(at, rng, n, ms, kv, lengths, caches)
        st = torch.cuda.current_stream().cuda_stream
        got = torch.full((n, H * hd), float("nan"), device="cuda")
        at.decode_batch_dev_noalloc(0, n, seqs.data_ptr(), pos.data_ptr(), max(lengths),
                                    q.data_ptr(), k.data_ptr(), v.data_ptr(), got.data_ptr(), st)
        torch.cuda.synchronize()
        got_np = got.cpu().numpy()
        kc = np.stack([c[0] for c in caches])
        vc = np.stack([c[1] for c in caches])
        tables = O.rope_tables(ms, hd, 500000.0)
        c = O.cfg(H, Hk, hd, ms)
        want = O.attn_decode_seqs(c, kc.reshape(-1), vc.reshape(-1), ms * kv,
                                  np.array(lengths, np.int32), q.cpu().numpy(),
                                  k.cpu().numpy(), v.cpu().numpy(), *tables,
                                  n_threads=os.cpu_count() or 1).reshape(n, H * hd)
        assert_attn_close(got_np, want, "capped no-alloc vs oracle")
        for s in (0, n // 2, n - 1):
            gk, gv = at.kv_download(s, 0, lengths[s], 1)
            np.testing.assert_array_equal(gk[0], kc[s, lengths[s]])
            np.testing.assert_array_equal(gv[0], vc[s, lengths[s]])
        # the allocating entry point on the same inputs (it re-appends the
        # same rows, so the output must not change)
        want_dev = torch.empty(n, H * hd, device="cuda")
        at.decode_batch_dev(0, n, seqs.data_ptr(), pos.data_ptr(), max(lengths), q.data_ptr(),
                            k.data_ptr(), v.data_ptr(), want_dev.data_ptr(), st)
        torch.cuda.synchronize()
        assert_attn_close(got_np, want_dev.cpu().numpy(), "capped no-alloc vs decode_batch_dev")


def test_noalloc_rejects_when_partial_slots_run_out():
    """300 sequences at head_dim 128 and 32 query heads: within the
    1024-sequence limit, but one slot per sequence already exceeds the 248
    that fit, so no slot is left for a CTA."""
    import torch
    H, Hk, hd, n = 32, 8, 128, 300
    assert SCRATCH_PART_BYTES // (H * (hd + 4) * 4) < n + 1
    with pb.Attn(1, H, Hk, 32, n_seqs=n, head_dim=hd) as at:
        d = torch.zeros(n * H * hd, device="cuda")
        idx = torch.arange(n, dtype=torch.int32, device="cuda")
        zero = torch.zeros(n, dtype=torch.int32, device="cuda")
        with pytest.raises(pb.PlAttnError) as ei:
            at.decode_batch_dev_noalloc(0, n, idx.data_ptr(), zero.data_ptr(), 0, d.data_ptr(),
                                        d.data_ptr(), d.data_ptr(), d.data_ptr())
        assert ei.value.rc == pb.PL_EARG
