"""The config-2 model file: our GGUF writer and Q4_K encoder (CPU only).

The encoder's blocks must decode, bit for bit, under picolm's own
dequantize_row_q4_K (quant.c:95-126) from the reference compiled here, and
picolm's own greedy driver must load and run the written file.
"""
import ctypes as C

import numpy as np
import pytest

from oracle import oracle as O
from oracle.make_gguf import make_model, q4k_decode, q4k_encode
from tests import e2e_util as E


def test_q4k_blocks_decode_identically_under_picolm():
    if not O.ref_available():
        pytest.skip("reference library oracle/_ref not built")
    lib = O.ref()
    lib.dequantize_row_q4_K.argtypes = [C.c_void_p, C.c_void_p, C.c_int]
    rng = np.random.default_rng(0)
    w = rng.standard_normal((6, 1024), dtype=np.float32) * np.float32(0.02)
    w[0, :256] = np.abs(w[0, :256])        # no negative values: zero offset
    w[1, :32] = 0.0                        # an all-zero sub-block
    w[2, 256:512] *= 40                    # a block with a large range
    data = q4k_encode(w, chunk_blocks=5)   # chunking must not change the bytes
    assert data == q4k_encode(w, chunk_blocks=10 ** 6)
    got = np.empty(w.size, np.float32)
    lib.dequantize_row_q4_K(C.create_string_buffer(data, len(data)), got.ctypes.data, w.size)
    np.testing.assert_array_equal(got, q4k_decode(data, w.size))
    # 4-bit quantisation: error within one step of each sub-block's range
    err = np.abs(got - w.ravel()).reshape(-1, 32)
    rng_sub = (np.maximum(w.reshape(-1, 32).max(1), 0) - np.minimum(w.reshape(-1, 32).min(1), 0))
    assert np.all(err.max(1) <= rng_sub / 15 * 0.75 + 1e-3 * np.abs(w).max())


def test_reference_driver_runs_a_written_model(tmp_path):
    if not E.have(E.E2E_REF):
        pytest.skip("oracle/_ref/e2e_ref not built (make -C oracle e2e)")
    path = str(tmp_path / "tiny.gguf")
    make_model(path, layers=2, dim=256, ffn=512, heads=4, kv_heads=2, vocab=1000, ctx=256)
    toks, margins, summary = E.run(E.E2E_REF, path, 16, 8)
    assert len(toks) == 8 and all(0 <= t < 1000 for t in toks)
    assert summary["prefill_tokens"] == 16
    # deterministic: the same file and seed give the same tokens
    assert E.run(E.E2E_REF, path, 16, 8)[0] == toks
