"""KV-axis split through the C ABI on one GPU (picolm_b200/shard.py).

One process plays both ranks of a 2-way split: rank r's rows live in cache
slot r of one context, the "gather" concatenates the two partials in rank
order, and pl_attn_combine_dev merges them.  The result must equal
picolm's unsplit decode chain (the oracle) within the attention tolerance,
and the appended rows must land, bit-exact, on the last rank only.
"""
import numpy as np
import pytest

from oracle import oracle as O
from tests.util import assert_attn_close, random_cache

pytestmark = pytest.mark.gpu

H, HK, HD = 32, 8, 64
KV_DIM = HK * HD
N_CACHED, N_NEW, WORLD = 3000, 4, 2


def test_two_rank_split_matches_unsplit_decode():
    import torch
    import picolm_b200 as pb
    from picolm_b200.shard import PART_STRIDE, AttnShardOps, KVSplitDecoder

    rng = np.random.default_rng(21)
    kc = random_cache(rng, N_CACHED, KV_DIM)
    vc = random_cache(rng, N_CACHED, KV_DIM)
    steps = [(rng.standard_normal(H * HD, dtype=np.float32),
              rng.standard_normal(KV_DIM, dtype=np.float32),
              rng.standard_normal(KV_DIM, dtype=np.float32)) for _ in range(N_NEW)]
    ms = N_CACHED + N_NEW
    dev = torch.device("cuda", 0)
    with pb.Attn(1, H, HK, ms, rope_base=500000.0, n_seqs=WORLD) as at:
        st = torch.cuda.current_stream(dev).cuda_stream
        decs = []
        for r in range(WORLD):
            d = KVSplitDecoder(rank=r, world=WORLD, n_cached=N_CACHED,
                               ops=AttnShardOps(at, st, seq=r))
            at.kv_upload(r, 0, 0, np.ascontiguousarray(kc[d.row0:d.row0 + d.n_rows]),
                         np.ascontiguousarray(vc[d.row0:d.row0 + d.n_rows]))
            decs.append(d)
        parts_all = torch.empty(WORLD * H * PART_STRIDE, device=dev)
        out = torch.empty(H * HD, device=dev)
        got = []
        for i, (q, k, v) in enumerate(steps):
            pos = N_CACHED + i
            qd, kd, vd = (torch.from_numpy(x).to(dev) for x in (q, k, v))
            for r, d in enumerate(decs):   # each "rank" writes its slice of the gather
                d.ops.partial(0, pos, d.row0, d.rows_at(pos), d.appends, qd, kd, vd,
                              parts_all[r * H * PART_STRIDE:(r + 1) * H * PART_STRIDE])
            decs[0].ops.combine(WORLD, parts_all, out)
            torch.cuda.synchronize()
            got.append(out.cpu().numpy().copy())
        # the appended rows are on the last rank only (local rows from n_rows)
        last = decs[-1]
        k_last, _ = at.kv_download(WORLD - 1, 0, 0, last.n_rows + N_NEW)
    fk = np.zeros((ms, KV_DIM), np.uint16)
    fv = np.zeros((ms, KV_DIM), np.uint16)
    fk[:N_CACHED], fv[:N_CACHED] = kc, vc
    tables = O.rope_tables(ms, HD, 500000.0)
    c = O.cfg(H, HK, HD, ms)
    for i, (q, k, v) in enumerate(steps):
        want, _, _ = O.attn_decode(c, fk.ravel(), fv.ravel(), N_CACHED + i, q, k, v, *tables)
        assert_attn_close(got[i], want, f"split step {i}")
    np.testing.assert_array_equal(k_last[last.n_rows:], fk[N_CACHED:])
    np.testing.assert_array_equal(k_last[:last.n_rows], kc[last.row0:])
