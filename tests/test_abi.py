"""The C-ABI library itself, without a GPU (CPU only).

libpl_attn.so must load on a host without a GPU, export every entry point
include/pl_attn.h declares, and answer without a device with a clean error
status (never a crash, never a CPU fallback).
"""
import ctypes as C
import subprocess

import numpy as np
import pytest

import picolm_b200 as pb


def test_library_builds_and_loads():
    from picolm_b200 import build
    build.build()
    lib = pb.load()
    assert lib is not None


def test_exports_every_declared_symbol():
    names = pb.declared_symbols()
    assert len(names) >= 15
    out = subprocess.run(["nm", "-D", "--defined-only", pb.LIB_PATH], check=True,
                         capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = [n for n in names if n not in exported]
    assert not missing, missing


def test_strerror_covers_every_code():
    lib = pb.load()
    for rc in range(0, -9, -1):
        s = lib.pl_attn_strerror(rc).decode()
        assert s and s != "unknown status"
    assert lib.pl_attn_strerror(-99).decode() == "unknown status"


def test_calls_before_init_report_state_error():
    lib = pb.load()
    assert lib.pl_attn_available() == 0
    q = np.zeros(2048, np.float32)
    k = np.zeros(256, np.float32)
    out = np.zeros(2048, np.float32)
    assert lib.pl_attn_decode(0, 0, 0, q, k, k, out) == pb.PL_ESTATE
    assert lib.pl_kv_download(0, 0, 0, 1, None, None) == pb.PL_ESTATE


def test_init_argument_checks_need_no_device():
    lib = pb.load()
    # unsupported head_dim / GQA ratios are rejected before any device call
    # (head_dim 64 and 128 are supported; 80, 96, 256 are not)
    for hd in (32, 80, 96, 256):
        assert lib.pl_attn_init(1, 32, 4, hd, 64, 1e4, 0, 1, 0) == pb.PL_EUNSUPPORTED
    assert lib.pl_attn_init(1, 48, 4, 64, 64, 1e4, 0, 1, 0) == pb.PL_EUNSUPPORTED
    assert lib.pl_attn_init(1, 32, 3, 64, 64, 1e4, 0, 1, 0) == pb.PL_EUNSUPPORTED
    assert lib.pl_attn_init(1, 16, 16, 64, 64, 1e4, 0, 1, 0) == pb.PL_EUNSUPPORTED
    assert lib.pl_attn_init(0, 32, 4, 64, 64, 1e4, 0, 1, 0) == pb.PL_EARG
    assert lib.pl_attn_init(1, 32, 4, 64, 64, 1e4, 7, 1, 0) == pb.PL_EARG


def test_init_without_device_fails_cleanly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(pb.PlAttnError) as ei:
        pb.Attn(1, 32, 4, 256)
    assert ei.value.rc == pb.PL_EDEVICE


def test_prefill_register_allocation_checked_at_build():
    """The build records ptxas' resource report and refuses a library whose
    prefill kernels would launch without the registers their warpgroup split
    (setmaxnreg) hands out."""
    import json
    from picolm_b200 import build
    build.build()
    res = json.load(open(build.RESOURCES))
    pf = {k: v for k, v in res.items() if "prefill_attn_kernel" in k}
    assert len(pf) == 2, sorted(pf)
    assert all(v["registers"] == build.PREFILL_LAUNCH_REGS for v in pf.values()), pf
    # the decode kernels at head_dim 64 run without spills
    dec64 = {k: v for k, v in res.items() if "decode_kernel" in k and k.endswith("Li64EEEvNS_10DecodeArgsE14CUtensorMap_stS2_")}
    assert dec64 and all(v.get("spill_stores", 0) == 0 for v in dec64.values()), dec64
    with pytest.raises(RuntimeError):
        build.check_resources({k: dict(v, registers=160) for k, v in pf.items()})
