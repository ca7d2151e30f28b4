"""Split by KV head: the decode of one sequence run as `world` head shards
(each with its own context holding all positions of its KV heads) equals the
unsharded decode.  The shards run one after another on one GPU here; on
several GPUs each rank runs one (bench.py, config 5)."""
import numpy as np
import pytest

import picolm_b200 as pb
from oracle import oracle as O
from picolm_b200.shard import head_shard
from tests.util import assert_attn_close, oracle_decode_layer, random_cache

pytestmark = pytest.mark.gpu

H, HK, HD = 32, 8, 64


@pytest.fixture(scope="module", autouse=True)
def _built():
    from picolm_b200 import build
    build.build()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_head_shards_equal_unsharded(world):
    rng = np.random.default_rng(50 + world)
    ms, P = 3000, 2900
    kv = HK * HD
    tables = O.rope_tables(ms, HD, 500000.0)
    kc, vc = random_cache(rng, ms, kv), random_cache(rng, ms, kv)
    q = rng.standard_normal(H * HD, dtype=np.float32)
    k = rng.standard_normal(kv, dtype=np.float32)
    v = rng.standard_normal(kv, dtype=np.float32)
    want, kc2, vc2 = oracle_decode_layer(H, HK, ms, kc, vc, P, q, k, v, tables)
    got = np.empty(H * HD, np.float32)
    for r in range(world):
        h0, hq, k0, hk = head_shard(H, HK, world, r)
        ks, ke = k0 * HD, (k0 + hk) * HD
        with pb.Attn(1, hq, hk, ms, rope_base=500000.0) as at:
            at.kv_upload(0, 0, 0, np.ascontiguousarray(kc[:, ks:ke]),
                         np.ascontiguousarray(vc[:, ks:ke]))
            got[h0 * HD:(h0 + hq) * HD] = at.decode(0, 0, P, q[h0 * HD:(h0 + hq) * HD],
                                                    k[ks:ke], v[ks:ke])
            gk, gv = at.kv_download(0, 0, P, 1)
        np.testing.assert_array_equal(gk[0], kc2[P, ks:ke])
        np.testing.assert_array_equal(gv[0], vc2[P, ks:ke])
    assert_attn_close(got, want, f"{world} head shards")
