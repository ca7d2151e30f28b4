"""KV-axis split over two GPUs with the merge over NVLink peer memory.

Two processes, one per GPU, each hold half of a sequence's cache; per
step each computes its partial and pl_attn_combine_p2p_dev pushes it to
the other GPU and merges (or, fused, pl_attn_decode_p2p_dev does both, the
merge grid pushing the partial itself).  With no cached rows, rank 0's
shard is empty and only takes part in the exchange.  Both ranks' outputs must equal picolm's
unsplit decode chain (the oracle) within the attention tolerance.  Needs
two GPUs (one process per GPU: the merge waits on the other rank).
"""
import os
import socket

import numpy as np
import pytest

from oracle import oracle as O
from tests.util import assert_attn_close, random_cache

pytestmark = pytest.mark.gpu

H, HK, HD = 32, 8, 64
KV_DIM = HK * HD
N_NEW, WORLD = 5, 2


def inputs(N_CACHED):
    rng = np.random.default_rng(31)
    kc = random_cache(rng, N_CACHED, KV_DIM)
    vc = random_cache(rng, N_CACHED, KV_DIM)
    steps = [(rng.standard_normal(H * HD, dtype=np.float32),
              rng.standard_normal(KV_DIM, dtype=np.float32),
              rng.standard_normal(KV_DIM, dtype=np.float32)) for _ in range(N_NEW)]
    return kc, vc, steps


def _rank_main(rank, world, port, out_dir, N_CACHED, fused):
    import torch
    import torch.distributed as dist
    import picolm_b200 as pb
    from picolm_b200.shard import PART_STRIDE, KVSplitDecoder, P2PShardOps
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        kc, vc, steps = inputs(N_CACHED)
        dev = torch.device("cuda", rank)
        with pb.Attn(1, H, HK, N_CACHED + N_NEW, rope_base=500000.0, device=rank) as at:
            st = torch.cuda.current_stream(dev).cuda_stream
            dec = KVSplitDecoder(rank=rank, world=world, n_cached=N_CACHED, ops=None)
            if dec.n_rows:
                at.kv_upload(0, 0, 0, np.ascontiguousarray(kc[dec.row0:dec.row0 + dec.n_rows]),
                             np.ascontiguousarray(vc[dec.row0:dec.row0 + dec.n_rows]))
            dec.ops = P2PShardOps(at, st, rank, world, fused=fused)
            part = torch.empty(H * PART_STRIDE, device=dev)
            out = torch.empty(H * HD, device=dev)
            outs = []
            for i, (q, k, v) in enumerate(steps):
                qd, kd, vd = (torch.from_numpy(x).to(dev) for x in (q, k, v))
                dec.step(0, N_CACHED + i, qd, kd, vd, part, None, out)
                torch.cuda.synchronize()
                outs.append(out.cpu().numpy().copy())
            np.save(os.path.join(out_dir, f"rank{rank}.npy"), np.stack(outs))
            dist.barrier()
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("N_CACHED", [3000, 0])
@pytest.mark.parametrize("fused", [True, False], ids=["decode_p2p", "combine_p2p"])
def test_two_gpu_p2p_split_matches_unsplit_decode(tmp_path, N_CACHED, fused):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs (one process per GPU)")
    mp.spawn(_rank_main, args=(WORLD, _free_port(), str(tmp_path), N_CACHED, fused),
             nprocs=WORLD, join=True)
    kc, vc, steps = inputs(N_CACHED)
    ms = N_CACHED + N_NEW
    fk = np.zeros((ms, KV_DIM), np.uint16)
    fv = np.zeros((ms, KV_DIM), np.uint16)
    fk[:N_CACHED], fv[:N_CACHED] = kc, vc
    tables = O.rope_tables(ms, HD, 500000.0)
    c = O.cfg(H, HK, HD, ms)
    want = []
    for i, (q, k, v) in enumerate(steps):
        w, _, _ = O.attn_decode(c, fk.ravel(), fv.ravel(), N_CACHED + i, q, k, v, *tables)
        want.append(w)
    for r in range(WORLD):
        got = np.load(tmp_path / f"rank{r}.npy")
        for i in range(N_NEW):
            assert_attn_close(got[i], want[i], f"rank {r} step {i}")
