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
import numpy as np
import pytest

import picolm_b200 as pb
from tests.util import assert_attn_close, random_cache

pytestmark = pytest.mark.gpu


def _setup(at, rng, n, ms, kv, lengths):
    import torch
    dev = torch.device("cuda", 0)
    for s in range(n):
        at.kv_upload(s, 0, 0, random_cache(rng, ms, kv), random_cache(rng, ms, kv))
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
