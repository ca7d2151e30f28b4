"""The NVLink exchange of a KV split (flag-in-data units, epoch parity, the
device-side merge counter) with one rank, on one GPU.

With world = 1 every merge block pushes its head into this rank's own
receive buffer and polls that same buffer, so no kernel waits for another
kernel or process: the single-GPU form of the path that
tests/test_shard_p2p_gpu.py runs over two GPUs.  Steps alternate between
pl_attn_decode_p2p_dev (the merge grid exchanges) and
pl_attn_decode_partial_dev + pl_attn_combine_p2p_dev (the exchange kernel),
so both forms share one epoch counter across more merges than the two
parity slots; one sequence is long enough for a split merge grid, the
other short enough for one CTA (the merge grid then pushes the CTA's
partial).  Every output must match picolm's unsplit decode (the oracle)
and every appended row its FP16 encoding.
"""
import numpy as np
import pytest

from oracle import oracle as O
from tests.util import assert_attn_close, random_cache

pytestmark = pytest.mark.gpu

H, HK, HD, LAYERS = 32, 8, 64, 2
KV_DIM = HK * HD
CACHED = (200, 10)  # rows already cached in slot 0 (split merge) and slot 1 (one CTA)
STEPS = 5


def test_one_rank_exchange_matches_unsplit_decode():
    import torch
    import picolm_b200 as pb

    rng = np.random.default_rng(61)
    ms = max(CACHED) + STEPS
    caches = {(s, l): (random_cache(rng, ms, KV_DIM), random_cache(rng, ms, KV_DIM))
              for s in range(len(CACHED)) for l in range(LAYERS)}
    tables = O.rope_tables(ms, HD, 500000.0)
    c = O.cfg(H, HK, HD, ms)
    dev = torch.device("cuda", 0)
    with pb.Attn(LAYERS, H, HK, ms, rope_base=500000.0, n_seqs=len(CACHED)) as at:
        for (s, l), (kc, vc) in caches.items():
            at.kv_upload(s, l, 0, kc[:CACHED[s]], vc[:CACHED[s]])
        h0 = at.xfer_setup(1, 0)
        at.xfer_connect([h0])
        st = torch.cuda.current_stream(dev).cuda_stream
        part = torch.empty(H * at.part_stride, device=dev)
        out = torch.empty(H * HD, device=dev)
        for step in range(STEPS):
            for s, n_cached in enumerate(CACHED):
                pos = n_cached + step
                for l in range(LAYERS):
                    q = rng.standard_normal(H * HD, dtype=np.float32)
                    k = rng.standard_normal(KV_DIM, dtype=np.float32)
                    v = rng.standard_normal(KV_DIM, dtype=np.float32)
                    qd, kd, vd = (torch.from_numpy(x).to(dev) for x in (q, k, v))
                    if (step + s) % 2 == 0:
                        at.decode_p2p_dev(s, l, pos, 0, pos + 1, 1, qd.data_ptr(), kd.data_ptr(),
                                          vd.data_ptr(), out.data_ptr(), st)
                    else:
                        at.decode_partial_dev(s, l, pos, 0, pos + 1, 1, qd.data_ptr(),
                                              kd.data_ptr(), vd.data_ptr(), part.data_ptr(), st)
                        at.combine_p2p_dev(part.data_ptr(), out.data_ptr(), st)
                    assert at.status(st) == pb.PL_OK
                    got = out.cpu().numpy()
                    kc, vc = caches[(s, l)]
                    want, _, _ = O.attn_decode(c, kc.ravel(), vc.ravel(), pos, q, k, v, *tables)
                    assert_attn_close(got, want, f"slot {s} layer {l} step {step}")
                    gk, gv = at.kv_download(s, l, pos, 1)
                    np.testing.assert_array_equal(np.ravel(gk), kc[pos])
                    np.testing.assert_array_equal(np.ravel(gv), vc[pos])


def test_one_rank_exchange_in_a_replayed_graph():
    """Captured once and replayed: the merges are numbered on the device, so
    every replay advances the epochs itself.  Re-running a step rewrites the
    same appended rows with the same values, so each replay must reproduce
    the first one bit for bit, and both must match the oracle."""
    import torch
    import picolm_b200 as pb

    rng = np.random.default_rng(62)
    n_cached, steps, ms = 300, 3, 320
    kc0 = random_cache(rng, ms, KV_DIM)
    vc0 = random_cache(rng, ms, KV_DIM)
    tables = O.rope_tables(ms, HD, 500000.0)
    c = O.cfg(H, HK, HD, ms)
    dev = torch.device("cuda", 0)
    qs = [rng.standard_normal(H * HD, dtype=np.float32) for _ in range(steps)]
    ks = [rng.standard_normal(KV_DIM, dtype=np.float32) for _ in range(steps)]
    vs = [rng.standard_normal(KV_DIM, dtype=np.float32) for _ in range(steps)]
    with pb.Attn(1, H, HK, ms, rope_base=500000.0) as at:
        at.kv_upload(0, 0, 0, kc0[:n_cached], vc0[:n_cached])
        at.xfer_connect([at.xfer_setup(1, 0)])
        qd = torch.from_numpy(np.stack(qs)).to(dev)
        kd = torch.from_numpy(np.stack(ks)).to(dev)
        vd = torch.from_numpy(np.stack(vs)).to(dev)
        out = torch.zeros(steps, H * HD, device=dev)

        def run(stream):
            for i in range(steps):
                pos = n_cached + i
                at.decode_p2p_dev(0, 0, pos, 0, pos + 1, 1, qd[i].data_ptr(), kd[i].data_ptr(),
                                  vd[i].data_ptr(), out[i].data_ptr(), stream)

        run(torch.cuda.current_stream(dev).cuda_stream)  # warm-up outside the capture
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            run(torch.cuda.current_stream(dev).cuda_stream)
        results = []
        for _ in range(3):
            out.zero_()
            graph.replay()
            torch.cuda.synchronize()
            results.append(out.cpu().numpy().copy())
        del graph
        assert at.status(torch.cuda.current_stream(dev).cuda_stream) == pb.PL_OK
    for r in results[1:]:
        np.testing.assert_array_equal(r.view(np.uint32), results[0].view(np.uint32))
    kc, vc = kc0.copy(), vc0.copy()
    for i in range(steps):
        want, _, _ = O.attn_decode(c, kc.ravel(), vc.ravel(), n_cached + i, qs[i], ks[i], vs[i],
                                   *tables)
        assert_attn_close(results[-1][i], want, f"replayed step {i}")
