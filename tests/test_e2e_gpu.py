"""End to end: picolm's greedy decoding with attention on the B200 (config 2).

The same driver (oracle/e2e_harness.c) is linked with picolm's own model.c
and with the copy whose attention blocks call this module.  On the same
random-init Q4_K model and prompt, the generated token ids must be
identical: every next-token argmax agrees.  A failure reports the first
divergent step and the top-2 logit margin there.

The full config-2 shape (22 layers, dim 2048, 128 + 128 tokens, ~620 MB
model) takes minutes of CPU time for the matmuls and runs only when
PL_E2E_FULL=1; its timings go to the JSON file named by PL_E2E_OUT.
"""
import json
import os

import pytest

from oracle.make_gguf import make_model
from tests import e2e_util as E

pytestmark = pytest.mark.gpu


def _need_binaries():
    if not (E.have(E.E2E_REF) and E.have(E.E2E_PL)):
        pytest.skip("oracle/_ref/e2e_ref / e2e_pl not built (make -C oracle e2e)")


def _compare(gguf, n_prompt, n_gen, threads):
    ref = E.run(E.E2E_REF, gguf, n_prompt, n_gen, threads=threads)
    ours = E.run(E.E2E_PL, gguf, n_prompt, n_gen, threads=threads)
    d = E.first_divergence(ref[0], ours[0])
    assert d is None, (f"greedy tokens diverge at step {d}: reference {ref[0][d]} "
                       f"(margin {ref[1][d]:.3g}), B200 attention {ours[0][d]} "
                       f"(margin {ours[1][d]:.3g})")
    return ref, ours


def test_greedy_tokens_identical_small_model(tmp_path):
    _need_binaries()
    path = str(tmp_path / "small.gguf")
    # 4 layers, 8 query / 2 KV heads of 64: the GQA shape of the configs
    make_model(path, layers=4, dim=512, ffn=1024, heads=8, kv_heads=2, vocab=2000, ctx=512)
    ref, ours = _compare(path, 96, 48, threads=4)
    assert len(ours[0]) == 48


def test_kv_cache_file_through_the_device(tmp_path):
    """kvcache_save / kvcache_load (model.c:1158-1259) with the cache in HBM.

    The KVCP file written by picolm with B200 attention has the reference's
    header and layer-0 rows bit-identical to the reference's (layer 0 sees
    identical inputs; RoPE and the FP16 append are bit-exact).  Deeper
    layers differ only through the attention outputs below them.  Loading
    the file into the device cache and saving it again reproduces it byte
    for byte, and generation after the load gives the same tokens."""
    import numpy as np
    _need_binaries()
    path = str(tmp_path / "small.gguf")
    make_model(path, layers=3, dim=512, ffn=1024, heads=8, kv_heads=2, vocab=2000, ctx=512)
    fa, fb, fc = (str(tmp_path / n) for n in ("ref.kv", "b200.kv", "roundtrip.kv"))
    ref = E.run(E.E2E_REF, path, 64, 16, save=fa)
    ours = E.run(E.E2E_PL, path, 64, 16, save=fb)
    ha, ka, va = E.read_kvcp(fa)
    hb, kb, vb = E.read_kvcp(fb)
    np.testing.assert_array_equal(ha, hb)
    np.testing.assert_array_equal(kb[0], ka[0])
    np.testing.assert_array_equal(vb[0], va[0])
    for x, y in ((ka, kb), (va, vb)):
        xf, yf = x.view(np.float16).astype(np.float32), y.view(np.float16).astype(np.float32)
        np.testing.assert_allclose(yf, xf, atol=2e-2, rtol=2e-2)
    again = E.run(E.E2E_PL, path, 64, 16, load=fb, save=fc)
    with open(fb, "rb") as f1, open(fc, "rb") as f2:
        assert f1.read() == f2.read(), "KVCP file changed on its way through the device cache"
    assert again[0] == ours[0], (again[0], ours[0])
    assert ref[0] == ours[0]


def test_block_greedy_tokens_identical_small_model(tmp_path):
    """The whole attention sub-block on the device (pl_attn_set_layer +
    pl_attn_block_prefill / pl_attn_block_decode): the projections sum in
    another order than picolm's, and the greedy tokens must still agree."""
    if not (E.have(E.E2E_REF) and E.have(E.E2E_BLK)):
        pytest.skip("oracle/_ref/e2e_ref / e2e_blk not built (make -C oracle e2e)")
    path = str(tmp_path / "small.gguf")
    make_model(path, layers=4, dim=512, ffn=1024, heads=8, kv_heads=2, vocab=2000, ctx=512)
    ref = E.run(E.E2E_REF, path, 96, 48, threads=4)
    blk = E.run(E.E2E_BLK, path, 96, 48, threads=4)
    d = E.first_divergence(ref[0], blk[0])
    assert d is None, (f"greedy tokens diverge at step {d}: reference {ref[0][d]} "
                       f"(margin {ref[1][d]:.3g}), B200 attention block {blk[0][d]} "
                       f"(margin {blk[1][d]:.3g})")


def test_greedy_tokens_identical_config2_full(tmp_path):
    if os.environ.get("PL_E2E_FULL") != "1":
        pytest.skip("full config 2 runs with PL_E2E_FULL=1 (minutes of CPU matmuls)")
    _need_binaries()
    path = str(tmp_path / "tinyllama_q4k.gguf")
    make_model(path)  # 22 layers, dim 2048, ffn 5632, 32/4 heads, vocab 32000, seed 1
    threads = min(16, os.cpu_count() or 1)
    ref, ours = _compare(path, 128, 128, threads=threads)
    blk = E.run(E.E2E_BLK, path, 128, 128, threads=threads) if E.have(E.E2E_BLK) else None
    out = os.environ.get("PL_E2E_OUT")
    if out:
        with open(out, "w") as f:
            json.dump({"threads": threads, "tokens_identical": len(ours[0]),
                       "min_margin": min(ref[1]), "reference": ref[2], "b200_attention": ours[2],
                       "b200_attention_block": blk[2] if blk else None,
                       "block_tokens_identical": (E.first_divergence(ref[0], blk[0]) is None
                                                  if blk else None),
                       "first_tokens": ours[0][:16]}, f, indent=1)
    if blk:
        d = E.first_divergence(ref[0], blk[0])
        assert d is None, f"attention block: greedy tokens diverge at step {d}"
