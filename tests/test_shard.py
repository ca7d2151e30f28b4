"""Host logic of the KV-axis split of one sequence (picolm_b200/shard.py).

Runs on the CPU: two gloo ranks each hold half of a sequence's cache and
decode three new tokens; their partials are all-gathered and merged, and
the result must equal picolm's unsplit attention (the oracle) within the
attention tolerance.  The partial/combine arithmetic here is a numpy
stand-in for the CUDA kernels (those are checked against the oracle in
tests/test_decode_gpu.py); what this test pins is the bookkeeping: shard
ranges, which rank appends, the rows each rank attends per step and the
rank order of the gather.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle as O
from picolm_b200.shard import PART_STRIDE, KVSplitDecoder, shard_range
from tests.util import ATOL, RTOL, random_cache

H, HK, HD = 8, 2, 64
KV_DIM = HK * HD
N_CACHED, N_NEW = 37, 3
LOG2E = 1.4426950408889634


def test_shard_range_covers_positions_in_rank_order():
    for n in (0, 1, 5, 64, 37, 32768, 32769):
        for world in (1, 2, 3, 4, 8):
            rows = []
            for r in range(world):
                row0, cnt = shard_range(n, world, r)
                assert cnt >= 0
                rows.extend(range(row0, row0 + cnt))
            assert rows == list(range(n)), (n, world)


def test_shard_range_rejects_bad_requests():
    with pytest.raises(ValueError):
        shard_range(10, 0, 0)
    with pytest.raises(ValueError):
        shard_range(10, 2, 2)


def test_rows_and_capacity_per_rank():
    last = KVSplitDecoder(rank=3, world=4, n_cached=100, ops=None)
    other = KVSplitDecoder(rank=1, world=4, n_cached=100, ops=None)
    assert (last.row0, last.n_rows, last.appends) == (75, 25, True)
    assert (other.row0, other.n_rows, other.appends) == (25, 25, False)
    assert last.rows_at(100) == 26 and last.rows_at(131) == 57
    assert other.rows_at(100) == 25 and other.rows_at(131) == 25
    assert last.local_capacity(32) == 57 and other.local_capacity(32) == 25
    with pytest.raises(ValueError):
        last.rows_at(99)


def rope_llama(x, pos, cos_t, sin_t):
    """picolm's pairwise RoPE (tensor.c:558-601): each product and the sum
    rounded separately, as the reference compiles without FMA."""
    x = np.asarray(x, np.float32).reshape(-1, HD)
    c = cos_t.reshape(-1, HD // 2)[pos]
    s = sin_t.reshape(-1, HD // 2)[pos]
    x0, x1 = x[:, 0::2], x[:, 1::2]
    y = np.empty_like(x)
    y[:, 0::2] = x0 * c - x1 * s
    y[:, 1::2] = x0 * s + x1 * c
    return y.ravel()


class NumpyShardOps:
    """CPU stand-in for pl_attn_decode_partial_dev / pl_attn_combine_dev."""

    def __init__(self, kc, vc, tables):
        self.kc, self.vc = kc, vc            # local cache rows, FP16 words
        self.cos, self.sin = tables

    def partial(self, layer, pos, row0, n_rows, append, q, k, v, part):
        qr = rope_llama(q, pos, self.cos, self.sin)
        if append:
            self.kc[pos - row0] = O.fp32_to_fp16(rope_llama(k, pos, self.cos, self.sin))
            self.vc[pos - row0] = O.fp32_to_fp16(v)
        K = O.fp16_to_fp32(self.kc[:n_rows]).reshape(n_rows, KV_DIM).astype(np.float64)
        V = O.fp16_to_fp32(self.vc[:n_rows]).reshape(n_rows, KV_DIM).astype(np.float64)
        part[:] = 0
        for h in range(H):
            kvh = h // (H // HK)
            base = h * PART_STRIDE
            if n_rows == 0:
                part[base] = -np.inf
                continue
            s = K[:, kvh * HD:(kvh + 1) * HD] @ qr[h * HD:(h + 1) * HD].astype(np.float64)
            s *= LOG2E / np.sqrt(HD)
            m = s.max()
            p = np.exp2(s - m)
            part[base] = m
            part[base + 1] = p.sum()
            part[base + 4:base + 4 + HD] = p @ V[:, kvh * HD:(kvh + 1) * HD]

    def gather(self, part, parts_all):
        chunks = [torch.empty_like(torch.from_numpy(part)) for _ in range(dist.get_world_size())]
        dist.all_gather(chunks, torch.from_numpy(part))
        parts_all[:] = torch.cat(chunks).numpy()

    def combine(self, world, parts_all, out):
        P = parts_all.reshape(world, H, PART_STRIDE)
        M = P[:, :, 0].max(axis=0)
        w = np.where(np.isneginf(P[:, :, 0]), 0.0, np.exp2(P[:, :, 0] - M))
        L = (w * P[:, :, 1]).sum(axis=0)
        O_ = (w[:, :, None] * P[:, :, 4:4 + HD]).sum(axis=0) / L[:, None]
        out[:] = O_.ravel()


def inputs():
    rng = np.random.default_rng(11)
    kc = random_cache(rng, N_CACHED, KV_DIM)
    vc = random_cache(rng, N_CACHED, KV_DIM)
    steps = [(rng.standard_normal(H * HD, dtype=np.float32),
              rng.standard_normal(KV_DIM, dtype=np.float32),
              rng.standard_normal(KV_DIM, dtype=np.float32)) for _ in range(N_NEW)]
    return kc, vc, steps


def _rank_main(rank, world, port, out_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        kc, vc, steps = inputs()
        tables = O.rope_tables(N_CACHED + N_NEW, HD, 10000.0)
        dec = KVSplitDecoder(rank=rank, world=world, n_cached=N_CACHED, ops=None)
        cap = dec.local_capacity(N_NEW)
        lk = np.zeros((cap, KV_DIM), np.uint16)
        lv = np.zeros((cap, KV_DIM), np.uint16)
        lk[:dec.n_rows] = kc[dec.row0:dec.row0 + dec.n_rows]
        lv[:dec.n_rows] = vc[dec.row0:dec.row0 + dec.n_rows]
        dec.ops = NumpyShardOps(lk, lv, tables)
        part = np.empty(H * PART_STRIDE, np.float64)
        parts_all = np.empty(world * H * PART_STRIDE, np.float64)
        outs = []
        for i, (q, k, v) in enumerate(steps):
            out = np.empty(H * HD, np.float64)
            dec.step(0, N_CACHED + i, q, k, v, part, parts_all, out)
            outs.append(out)
        if rank == 0:
            np.save(out_path, np.stack(outs))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2])
def test_split_decode_equals_unsplit_attention(tmp_path, world):
    out_path = str(tmp_path / "split.npy")
    mp.spawn(_rank_main, args=(world, _free_port(), out_path), nprocs=world, join=True)
    got = np.load(out_path)
    # the unsplit reference: picolm's decode chain on the whole cache
    kc, vc, steps = inputs()
    ms = N_CACHED + N_NEW
    fk = np.zeros((ms, KV_DIM), np.uint16)
    fv = np.zeros((ms, KV_DIM), np.uint16)
    fk[:N_CACHED], fv[:N_CACHED] = kc, vc
    tables = O.rope_tables(ms, HD, 10000.0)
    c = O.cfg(H, HK, HD, ms)
    for i, (q, k, v) in enumerate(steps):
        want, _, _ = O.attn_decode(c, fk.ravel(), fv.ravel(), N_CACHED + i, q, k, v, *tables)
        np.testing.assert_allclose(got[i], want, atol=ATOL, rtol=RTOL)


def test_head_shard_covers_heads_in_rank_order():
    from picolm_b200.shard import head_shard
    for H_, Hk_ in ((32, 8), (32, 4), (8, 8), (16, 2)):
        for world in (1, 2, 4, 8):
            if Hk_ % world:
                with pytest.raises(ValueError):
                    head_shard(H_, Hk_, world, 0)
                continue
            q_heads, kv_heads = [], []
            for r in range(world):
                h0, hq, k0, hk = head_shard(H_, Hk_, world, r)
                assert hq == hk * (H_ // Hk_)
                assert h0 == k0 * (H_ // Hk_)   # query heads stay with their KV head
                q_heads.extend(range(h0, h0 + hq))
                kv_heads.extend(range(k0, k0 + hk))
            assert q_heads == list(range(H_)) and kv_heads == list(range(Hk_))
