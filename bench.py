#!/usr/bin/env python
"""bench.py -- picolm attention hot path on B200 (one JSON line on rank 0).

Headline workload ("config 4"): batched decode,
64 independent sequences per GPU, 2048 cached positions each, TinyLlama
heads (32 query / 4 KV, head_dim 64), one new token per sequence per step;
the config's 64 decode steps (positions 2048..2111), cycled.  A step is one
call of pl_attn_decode_batch_dev (one fused kernel: RoPE + FP16 append +
split-KV attention + merge).  Four disjoint sets of 64 sequences take the
steps in turn, so that each step reads 134 MB of cache the previous three
did not touch (more than the 126 MB L2, in place of a flush), and the timed
steps run back to back.

  metric  decode-attn HBM GB/s = algorithmic bytes / device time, summed
          over all ranks (KV rows read + q/k/v read + KV row and output
          written; bytes per step in step_bytes())
  e2e     the same metric through the host-buffer C entry point
          pl_attn_decode_batch (pinned staging, H2D of q/k/v, D2H of out,
          synchronous), i.e. what a C caller of the library sees
  extra   prefill (config 3: causal prefill S=2048, 22 layers, TFLOPS),
          long_ctx (config 5: 32768 cached, 16 layers, 32 steps, GB/s),
          decode1 (config 1: one TinyLlama decode layer at pos 255, us/call)
          -- single-GPU runs only.

Multi-GPU: one process per GPU (torchrun); sequences are independent, so
each rank runs its own 64 sequences with no collective on the data path
(weak scaling); timing is the max over ranks of the device time.

`--impl reference` times picolm's own CPU attention (oracle/_ref: the
reference sources compiled in place; else the C restatement) on the same
workload and prints the same line with "impl": "reference".
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

H, HK, HD = 32, 4, 64          # TinyLlama heads
SEQS_PER_GPU = 64
CTX = 2048
NSTEP = 64                     # positions 2048 .. 2111
KV_DIM = HK * HD
Q_DIM = H * HD
L2_FLUSH_BYTES = 256 << 20     # > 126 MB L2
KV_SETS = 4                    # disjoint sets of SEQS_PER_GPU sequences used in rotation


def step_bytes(pos: int, n_seq: int) -> int:
    """Algorithmic bytes of one decode step for n_seq sequences at pos."""
    rows = pos + 1
    per_seq = (rows * KV_DIM * 2 * 2          # K and V rows read (FP16)
               + Q_DIM * 4 + 2 * KV_DIM * 4   # q, k, v read (FP32)
               + 2 * KV_DIM * 2               # appended K and V row (FP16)
               + Q_DIM * 4)                   # output (FP32)
    return per_seq * n_seq


def load_peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def profile_traffic(name: str):
    """Per-launch DRAM bytes recorded in profiles/<name> ('traffic_bytes_per_launch: N')."""
    p = os.path.join(ROOT, "profiles", name)
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.startswith("traffic_bytes_per_launch:"):
            return float(line.split(":", 1)[1])
    return None


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """NVML samples of SM clock and throttle reasons while a region runs."""
    HW_SLOW, SW_THERM, HW_THERM, SW_POWER = 0x8, 0x20, 0x40, 0x4

    def __init__(self, cuda_index: int):
        self.samples, self.reasons, self.max_mhz = [], 0, None
        self._stop = threading.Event()
        self._h = None
        try:
            import pynvml
            pynvml.nvmlInit()
            import torch
            p = torch.cuda.get_device_properties(cuda_index)
            # torch reports the PCI location as integers; NVML wants the
            # "domain:bus:device.function" string
            bus = f"{int(p.pci_domain_id):08X}:{int(p.pci_bus_id):02X}:{int(p.pci_device_id):02X}.0"
            try:
                self._h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            except Exception:
                self._h = pynvml.nvmlDeviceGetHandleByIndex(cuda_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self._nv = pynvml
        except Exception:
            self._h = None

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                self.reasons |= nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
            except Exception:
                pass
            # the timed regions are short (about 0.6 ms for 20 decode steps):
            # sample as often as NVML answers
            time.sleep(0.0005)

    def __enter__(self):
        if self._h is not None:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *exc):
        if self._h is not None:
            self._stop.set()
            self._t.join()

    def summary(self) -> dict:
        names = []
        for bit, name in ((self.HW_SLOW, "hw_slowdown"), (self.SW_THERM, "sw_thermal_slowdown"),
                          (self.HW_THERM, "hw_thermal_slowdown"), (self.SW_POWER, "sw_power_cap")):
            if self.reasons & bit:
                names.append(name)
        return {"sm_mhz": float(np.median(self.samples)) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": names, "samples": len(self.samples)}


# ------------------------------------------------------------ distributed
def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    import torch
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return rank, world, local


def per_rank(x: float, world: int) -> list:
    """x of every rank, in rank order (a list of one on a single GPU)."""
    if world == 1:
        return [x]
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    out = [torch.zeros_like(t) for _ in range(world)]
    dist.all_gather(out, t)
    return [float(v.item()) for v in out]


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


# ------------------------------------------------------------ workloads
def make_cache_host(rng, n_rows: int, kv_dim: int) -> np.ndarray:
    x = rng.standard_normal((n_rows, kv_dim), dtype=np.float32)
    return x.astype(np.float16).view(np.uint16)


def run_batched_decode(args, rank, world, local, peaks):
    """The headline: KV_SETS disjoint sets of SEQS_PER_GPU sequences (134 MB
    of cache each, 2048 rows per sequence) used in rotation, one set per
    step, so every step reads 134 MB that the previous KV_SETS - 1 steps
    (402 MB) did not touch -- inputs larger than the 126 MB L2, as the
    timing rules allow in place of a flush.  The K timed steps run back to
    back between one barrier + synchronize pair.  Set k's j-th step appends
    and attends at position CTX + j mod NSTEP."""
    import torch
    import picolm_b200 as pb
    dev = torch.device("cuda", local)
    n_slots = SEQS_PER_GPU * KV_SETS
    at = pb.Attn(1, H, HK, CTX + NSTEP, n_seqs=n_slots, device=local)
    rng = np.random.default_rng(3 + 1000 * rank)
    for s in range(n_slots):
        at.kv_upload(s, 0, 0, make_cache_host(rng, CTX, KV_DIM), make_cache_host(rng, CTX, KV_DIM))
    gen = torch.Generator(device=dev).manual_seed(3 + rank)
    q = torch.randn(NSTEP, SEQS_PER_GPU, Q_DIM, device=dev, generator=gen)
    k = torch.randn(NSTEP, SEQS_PER_GPU, KV_DIM, device=dev, generator=gen)
    v = torch.randn(NSTEP, SEQS_PER_GPU, KV_DIM, device=dev, generator=gen)
    out = torch.empty(NSTEP, SEQS_PER_GPU, Q_DIM, device=dev)
    seqs = [torch.arange(ks * SEQS_PER_GPU, (ks + 1) * SEQS_PER_GPU, dtype=torch.int32, device=dev)
            for ks in range(KV_SETS)]
    pos = (CTX + torch.arange(NSTEP, dtype=torch.int32, device=dev))[:, None].repeat(
        1, SEQS_PER_GPU).contiguous()
    stream = torch.cuda.current_stream(dev)
    sh = stream.cuda_stream

    def step_pos(i):
        return (i // KV_SETS) % NSTEP

    def step(i):
        s = step_pos(i)
        at.decode_batch_dev(0, SEQS_PER_GPU, seqs[i % KV_SETS].data_ptr(), pos[s].data_ptr(),
                            CTX + NSTEP - 1, q[s].data_ptr(), k[s].data_ptr(), v[s].data_ptr(),
                            out[s].data_ptr(), sh)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    total_bytes = sum(step_bytes(CTX + step_pos(args.warmup + j), SEQS_PER_GPU)
                      for j in range(args.steps))
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        t0.record(stream)
        for j in range(args.steps):
            step(args.warmup + j)
        t1.record(stream)
        torch.cuda.synchronize()
    barrier(world)
    # the decode kernel in isolation: a second pass with the module's own
    # CUDA events around each decode launch.  An event between two launches
    # stops the next decode grid from running its set-up under the tail of
    # the kernel before it (programmatic dependent launch), so this pass
    # times each launch with its set-up exposed; it is reported beside the
    # roofline, which uses the timed region above.
    n_prof = min(args.steps, 256)
    at.profile(True)
    prof_bytes = 0
    for j in range(n_prof):
        i = args.warmup + j
        step(i)
        prof_bytes += step_bytes(CTX + step_pos(i), SEQS_PER_GPU)
    torch.cuda.synchronize()
    kern_ms, n_attn, n_all = at.profile_read()
    at.profile(False)
    launches_per_step = n_all / n_prof
    t_local = t0.elapsed_time(t1) / 1e3
    t_ranks = per_rank(t_local, world)
    t_max = max(t_ranks)
    value = total_bytes * world / t_max / 1e9
    isolated = prof_bytes / (kern_ms / 1e3) / 1e9     # per launch bytes / isolated launch time
    # One decode launch per step: bytes per launch over the timed region's
    # average step, which also holds the step's merge launch, so a lower
    # bound on the decode kernel's own rate in the back-to-back loop.
    achieved = total_bytes / t_local / 1e9
    res = {
        "value": value, "ms_per_step": t_max * 1e3 / args.steps,
        "rank_ms_per_step": [t * 1e3 / args.steps for t in t_ranks],
        "tok_per_s": SEQS_PER_GPU * world * args.steps / t_max,
        "pct_peak": 100.0 * value / world / peaks["hbm_gbs"],
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"],
                     "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"],
                     "peak_source": peaks["source"] + " (hbm_gbs, burst copy)",
                     "traffic": profile_traffic("decode_kernel_config4.txt"),
                     "kernel": "pl::decode_kernel<32,4> (fused RoPE + append + split-KV "
                               "attention; the split merge is a second, PDL-overlapped kernel)",
                     "timing": "CUDA events around the timed region's back-to-back steps, "
                               "one decode + one merge launch per step (the merge's time is "
                               "counted against the decode kernel)",
                     "isolated_launch_gbs": isolated,
                     "isolated_launch_frac": isolated / peaks["hbm_gbs"],
                     "bytes_per_launch": total_bytes / args.steps},
        "gpu_launches": int(round(launches_per_step * args.steps)),
        "launches_per_step": launches_per_step, "clocks": clk.summary(),
    }
    # ---- end to end through the host-buffer C entry point
    qh = q.cpu().numpy()
    kh = k.cpu().numpy()
    vh = v.cpu().numpy()
    seqs_h = [np.arange(ks * SEQS_PER_GPU, (ks + 1) * SEQS_PER_GPU, dtype=np.int32)
              for ks in range(KV_SETS)]
    out_h = np.empty(SEQS_PER_GPU * Q_DIM, np.float32)  # reused, like model.c's s->xb
    n_e2e = max(64, min(args.steps, 256))
    for i in range(3):
        at.decode_batch(0, seqs_h[i % KV_SETS], np.full(SEQS_PER_GPU, CTX + NSTEP - 1, np.int32),
                        qh[0], kh[0], vh[0], out=out_h)
    # the C entry point through a plain void* binding (what a C caller or a
    # thin FFI stub pays per call; numpy argument conversion is left out)
    raw = at.raw().pl_attn_decode_batch
    pos_h = [np.full(SEQS_PER_GPU, CTX + s, np.int32) for s in range(NSTEP)]
    call_args = [(seqs_h[j % KV_SETS].ctypes.data, pos_h[step_pos(j)].ctypes.data,
                  qh[step_pos(j)].ctypes.data, kh[step_pos(j)].ctypes.data,
                  vh[step_pos(j)].ctypes.data, out_h.ctypes.data) for j in range(n_e2e)]

    def e2e_loop():
        nbytes = 0
        barrier(world)
        t0 = time.perf_counter()
        for j in range(n_e2e):
            rc = raw(0, SEQS_PER_GPU, *call_args[j])
            if rc:
                raise pb.PlAttnError(rc, "pl_attn_decode_batch")
            nbytes += step_bytes(CTX + step_pos(j), SEQS_PER_GPU)
        return nbytes, max_over_ranks(time.perf_counter() - t0, world)

    # the caller's buffers through the staging area, then registered once
    # (pl_attn_host_register, as model.c would register s->q/k/v/xb at start-up)
    _, t_staged = e2e_loop()
    registered = register_all(at, (qh, kh, vh, out_h))
    e2e_bytes, t_e2e = e2e_loop()
    for arr in registered:
        at.host_unregister(arr)
    h2d = SEQS_PER_GPU * (Q_DIM + 2 * KV_DIM) * 4 + 2 * SEQS_PER_GPU * 4
    d2h = SEQS_PER_GPU * Q_DIM * 4 + 4
    call_us = t_e2e * 1e6 / n_e2e
    # where a call's time goes: q to the device (for comparison, a pinned-to-
    # device copy of the same bytes, timed alone with CUDA events), the
    # decode + merge launches as timed one by one above (the merge then
    # writes the output over the bus instead), and the rest: the small copy
    # of slots and positions, k/v read and the output written over the bus,
    # launch and wake-up latency, host work
    qpin = torch.empty(SEQS_PER_GPU * Q_DIM, dtype=torch.float32, pin_memory=True)
    qdev = torch.empty(SEQS_PER_GPU * Q_DIM, dtype=torch.float32, device=dev)
    for _ in range(3):
        qdev.copy_(qpin, non_blocking=True)
    c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    c0.record()
    for _ in range(20):
        qdev.copy_(qpin, non_blocking=True)
    c1.record()
    torch.cuda.synchronize()
    h2d_q_us = c0.elapsed_time(c1) * 1e3 / 20
    kern_us = kern_ms * 1e3 / n_prof
    res["e2e"] = {"value": e2e_bytes * world / t_e2e / 1e9, "unit": "GB/s",
                  "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                  "ms_per_step": t_e2e * 1e3 / n_e2e, "steps": n_e2e,
                  "api": "pl_attn_decode_batch through a void* ctypes binding (host "
                         "buffers registered with pl_attn_host_register, synchronous)",
                  "phases_us": {"call": call_us, "h2d_q_copy": h2d_q_us,
                                "decode_merge_launches": kern_us,
                                "rest": call_us - h2d_q_us - kern_us},
                  "path": "no copies: q read over the bus into HBM by a gather kernel that the "
                          "decode grid queues behind (programmatic dependent launch), slots and "
                          "positions in the kernel arguments, k and v read by the appending "
                          "segment and the output written by the merge over the bus from / into "
                          "the registered buffers",
                  "unregistered_ms_per_step": t_staged * 1e3 / n_e2e}
    at.close()
    return res


def register_all(at, arrays):
    """Page-lock the host arrays of an end-to-end loop; an array the driver
    refuses stays on the staging path (the call still works)."""
    import picolm_b200 as pb
    done = []
    for arr in arrays:
        try:
            at.host_register(arr)
            done.append(arr)
        except pb.PlAttnError as e:
            print(f"bench: host_register refused ({e}); that array is staged", file=sys.stderr)
    return done


def cpu_decode_sample(max_seconds: float = 15.0, n_threads: int | None = None,
                      steps: int | None = None, warmup: int = 0):
    """picolm's CPU attention on the config-4 workload: full decode steps of
    all 64 sequences (2048+ cached rows each), independent sequences spread
    over the host's threads.  With `steps`, `warmup` untimed steps and then
    exactly `steps` timed ones (the reference arm); else timed steps until
    ~max_seconds of work."""
    from oracle import oracle as O
    use_ref = O.ref_available()
    n_threads = n_threads or os.cpu_count() or 1
    rng = np.random.default_rng(3)
    ms = CTX + NSTEP
    kc = np.zeros((SEQS_PER_GPU, ms, KV_DIM), np.uint16)
    vc = np.zeros((SEQS_PER_GPU, ms, KV_DIM), np.uint16)
    for s in range(SEQS_PER_GPU):
        kc[s, :CTX] = make_cache_host(rng, CTX, KV_DIM)
        vc[s, :CTX] = make_cache_host(rng, CTX, KV_DIM)
    kf, vf = kc.reshape(-1), vc.reshape(-1)
    c = O.cfg(H, HK, HD, ms)
    tables = O.rope_tables(ms, HD, 10000.0)
    def one_step(j):
        p = CTX + j % NSTEP  # the config's 64 positions, cycled like the GPU arm
        q = rng.standard_normal(SEQS_PER_GPU * Q_DIM, dtype=np.float32)
        k = rng.standard_normal(SEQS_PER_GPU * KV_DIM, dtype=np.float32)
        v = rng.standard_normal(SEQS_PER_GPU * KV_DIM, dtype=np.float32)
        O.attn_decode_seqs(c, kf, vf, ms * KV_DIM, np.full(SEQS_PER_GPU, p, np.int32), q, k, v,
                           *tables, n_threads=n_threads, use_ref=use_ref)
        return step_bytes(p, SEQS_PER_GPU)

    for j in range(warmup):
        one_step(j)
    total_bytes, n = 0, 0
    t0 = time.perf_counter()
    while (n < steps) if steps is not None else (n < NSTEP):
        total_bytes += one_step(warmup + n)
        n += 1
        if steps is None and time.perf_counter() - t0 > max_seconds:
            break
    dt = time.perf_counter() - t0
    return {"value": total_bytes / dt / 1e9, "unit": "GB/s", "cores": n_threads,
            "kind": "reference" if use_ref else "port", "steps": n,
            "sample": f"{n} full decode steps x {SEQS_PER_GPU} seqs at positions {CTX}.."
                      f"{CTX + NSTEP - 1} cycled (config 4), {n_threads} threads, one sequence "
                      f"per thread at a time (picolm's attention loop is single-threaded)",
            "s_per_step": dt / n}


def cpu_config1_sample(max_seconds: float = 3.0):
    """picolm's CPU attention on config 1: one TinyLlama decode layer at
    position 255 (255 cached rows), one call at a time on one thread, as
    model_forward_ex runs it."""
    from oracle import oracle as O
    use_ref = O.ref_available()
    rng = np.random.default_rng(0)
    ms = 256
    kc0 = np.zeros((ms, KV_DIM), np.uint16)
    vc0 = np.zeros((ms, KV_DIM), np.uint16)
    kc0[:255] = make_cache_host(rng, 255, KV_DIM)
    vc0[:255] = make_cache_host(rng, 255, KV_DIM)
    c = O.cfg(H, HK, HD, ms)
    tables = O.rope_tables(ms, HD, 10000.0)
    q = rng.standard_normal(Q_DIM, dtype=np.float32)
    k = rng.standard_normal(KV_DIM, dtype=np.float32)
    v = rng.standard_normal(KV_DIM, dtype=np.float32)
    pos = np.array([255], np.int32)
    kc, vc = kc0.ravel().copy(), vc0.ravel().copy()
    n, t_sum = 0, 0.0
    while t_sum < max_seconds or n < 3:
        qq, kk = q.copy(), k.copy()  # the loop rotates q and k in place
        t0 = time.perf_counter()
        O.attn_decode_seqs(c, kc, vc, ms * KV_DIM, pos, qq, kk, v, *tables, n_threads=1,
                           use_ref=use_ref)
        t_sum += time.perf_counter() - t0
        n += 1
    return {"value": t_sum / n * 1e6, "unit": "us per call", "cores": 1,
            "kind": "reference" if use_ref else "port",
            "sample": f"{n} calls of one decode layer at position 255 (config 1), one thread "
                      f"(picolm's attention loop is single-threaded)"}


def cpu_prefill_sample(n_threads: int | None = None):
    """picolm's CPU attention on config 3: full causal prefills of 2048
    positions, each layer's positions one after another on one thread (as
    model_forward_prefill runs them), independent layers on separate host
    threads -- one full layer per thread, min(threads, 22) layers."""
    from oracle import oracle as O
    use_ref = O.ref_available()
    n_threads = n_threads or os.cpu_count() or 1
    L, S = min(n_threads, 22), 2048
    rng = np.random.default_rng(2)
    kc = np.zeros(L * S * KV_DIM, np.uint16)
    vc = np.zeros(L * S * KV_DIM, np.uint16)
    q = rng.standard_normal((L, S, Q_DIM), dtype=np.float32).astype(np.float16).astype(np.float32)
    k = rng.standard_normal((L, S, KV_DIM), dtype=np.float32).astype(np.float16).astype(np.float32)
    v = rng.standard_normal((L, S, KV_DIM), dtype=np.float32).astype(np.float16).astype(np.float32)
    c = O.cfg(H, HK, HD, S)
    tables = O.rope_tables(S, HD, 10000.0)
    t0 = time.perf_counter()
    O.attn_prefill_seqs(c, kc, vc, S * KV_DIM, 0, S, q, k, v, *tables, n_threads=L,
                        use_ref=use_ref)
    dt = time.perf_counter() - t0
    flops = 4.0 * H * HD * S * (S + 1) / 2
    return {"value": flops * L / dt / 1e12, "unit": "TFLOP/s", "cores": L,
            "kind": "reference" if use_ref else "port",
            "s_per_layer": dt, "layers_per_s": L / dt,
            "sample": f"{L} full causal prefill layers of 2048 positions (config 3), one layer "
                      f"per thread on {L} threads; s_per_layer is one layer's time on one "
                      f"thread (measured, not extrapolated)"}


def cpu_long_ctx_sample(max_seconds: float = 12.0, n_threads: int | None = None):
    """picolm's CPU attention on config 5: decode steps of one sequence with
    32768 cached rows over 16 layers (32/8 heads, theta 5e5); the 16 layers
    of a step are independent here and run on separate host threads, each
    layer's loop on one thread as in picolm."""
    from oracle import oracle as O
    use_ref = O.ref_available()
    n_threads = n_threads or os.cpu_count() or 1
    L, HK5, CTX5, NS5 = 16, 8, 32768, 32
    kv5 = HK5 * HD
    ms = CTX5 + NS5
    rng = np.random.default_rng(4)
    kc = np.zeros((L, ms, kv5), np.uint16)
    vc = np.zeros((L, ms, kv5), np.uint16)
    # one layer's rows, copied to all 16 (the loop's time does not depend on
    # the values; this keeps the set-up short)
    kc[:, :CTX5] = make_cache_host(rng, CTX5, kv5)
    vc[:, :CTX5] = make_cache_host(rng, CTX5, kv5)
    kf, vf = kc.reshape(-1), vc.reshape(-1)
    c = O.cfg(H, HK5, HD, ms)
    tables = O.rope_tables(ms, HD, 500000.0)
    total, steps = 0, 0
    t0 = time.perf_counter()
    while steps < NS5:
        p = CTX5 + steps
        q = rng.standard_normal(L * Q_DIM, dtype=np.float32)
        k = rng.standard_normal(L * kv5, dtype=np.float32)
        v = rng.standard_normal(L * kv5, dtype=np.float32)
        O.attn_decode_seqs(c, kf, vf, ms * kv5, np.full(L, p, np.int32), q, k, v, *tables,
                           n_threads=min(n_threads, L), use_ref=use_ref)
        total += L * ((p + 1) * kv5 * 4 + Q_DIM * 8 + kv5 * 12)
        steps += 1
        if time.perf_counter() - t0 > max_seconds:
            break
    dt = time.perf_counter() - t0
    return {"value": total / dt / 1e9, "unit": "GB/s", "cores": min(n_threads, L),
            "kind": "reference" if use_ref else "port", "ms_per_step_16_layers": dt / steps * 1e3,
            "sample": f"{steps} decode steps (16 layers each) at positions {CTX5}.."
                      f"{CTX5 + steps - 1} (config 5), layers on {min(n_threads, L)} threads"}


def run_prefill(args, local, peaks):
    """Config 3: causal prefill, S=2048, 22 layers back to back."""
    import torch
    import picolm_b200 as pb
    L, S = 22, 2048
    dev = torch.device("cuda", local)
    at = pb.Attn(L, H, HK, S, device=local)
    gen = torch.Generator(device=dev).manual_seed(2)
    # Q, K, V FP16-valued ~N(0,1), handed over as FP32 (model.c's q_batch etc.)
    q = torch.randn(L, S, Q_DIM, device=dev, generator=gen).half().float()
    k = torch.randn(L, S, KV_DIM, device=dev, generator=gen).half().float()
    v = torch.randn(L, S, KV_DIM, device=dev, generator=gen).half().float()
    out = torch.empty(L, S, Q_DIM, device=dev)
    sh = torch.cuda.current_stream(dev).cuda_stream
    flops_layer = 4.0 * H * HD * S * (S + 1) / 2

    def run_all():
        for l in range(L):
            at.prefill_dev(0, l, 0, S, q[l].data_ptr(), k[l].data_ptr(), v[l].data_ptr(),
                           out[l].data_ptr(), None, sh)

    for _ in range(3):
        run_all()
    torch.cuda.synchronize()
    # whole calls as a caller sees them (the attention grid overlaps the
    # prologue through programmatic dependent launch)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 5
    e0.record()
    for _ in range(reps):
        run_all()
    e1.record()
    torch.cuda.synchronize()
    total_ms = e0.elapsed_time(e1)
    # the attention kernel alone: the module's events around each launch
    # (they separate it from the prologue)
    at.profile(True)
    for _ in range(reps):
        run_all()
    torch.cuda.synchronize()
    kern_ms, n_attn, n_all = at.profile_read()
    at.profile(False)
    tflops_kernel = flops_layer * L * reps / (kern_ms / 1e3) / 1e12
    res = {"metric": "prefill-attn TFLOPS (causal FLOPs / attention-kernel time)",
           "value": tflops_kernel, "unit": "TFLOP/s",
           "config": {"workload": "config3 causal prefill S=2048 x 22 layers, 32/4 heads, hd 64, "
                                  "Q/K/V fp16-valued N(0,1) seed 2"},
           "ms_per_22_layers": total_ms / reps,
           "attn_kernel_ms_per_layer": kern_ms / (L * reps),
           "tflops_whole_call": flops_layer * L * reps / (total_ms / 1e3) / 1e12,
           "roofline": {"bound": "tensor", "achieved": tflops_kernel,
                        "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                        "frac": tflops_kernel / peaks["bf16_tflops"],
                        "peak_source": peaks["source"] + " (bf16 dense burst; fp16 taken equal)",
                        "traffic": profile_traffic("prefill_attn_kernel_config3.txt"),
                        "kernel": "pl::prefill_attn_kernel (tcgen05, TMEM accumulators, TMA)",
                        "flops_per_launch": flops_layer},
           "gpu_launches": n_all}
    # end to end through the host-buffer entry point, one layer
    qh, kh, vh = q[0].cpu().numpy(), k[0].cpu().numpy(), v[0].cpu().numpy()
    out_h = np.empty(S * Q_DIM, np.float32)  # reused, like model.c's xb_batch
    at.prefill(0, 0, 0, qh, kh, vh, out=out_h)
    n = 5

    def e2e_loop():
        t0 = time.perf_counter()
        for _ in range(n):
            at.prefill(0, 0, 0, qh, kh, vh, out=out_h)
        return (time.perf_counter() - t0) / n

    dt_staged = e2e_loop()
    registered = register_all(at, (qh, kh, vh, out_h))
    dt = e2e_loop()
    for arr in registered:
        at.host_unregister(arr)
    res["e2e"] = {"value": flops_layer / dt / 1e12, "unit": "TFLOP/s",
                  "h2d_bytes_per_step": S * (Q_DIM + 2 * KV_DIM) * 4,
                  "d2h_bytes_per_step": S * Q_DIM * 4 + 4, "ms_per_layer": dt * 1e3,
                  "api": "pl_attn_prefill (host buffers registered with pl_attn_host_register)",
                  "unregistered_ms_per_layer": dt_staged * 1e3}
    at.close()
    return res


def run_long_ctx(args, local, peaks):
    """Config 5 on one GPU: 16 layers, 32/8 heads, 32768 cached, 32 steps."""
    import torch
    import picolm_b200 as pb
    L, HK5, CTX5, NS5 = 16, 8, 32768, 32
    kv5 = HK5 * HD
    dev = torch.device("cuda", local)
    at = pb.Attn(L, H, HK5, CTX5 + NS5, rope_base=500000.0, device=local)
    rng = np.random.default_rng(4)
    # one layer's rows uploaded to all 16 layers (each layer its own HBM
    # slab; the kernels' time does not depend on the values), which keeps
    # the set-up short
    kc5, vc5 = make_cache_host(rng, CTX5, kv5), make_cache_host(rng, CTX5, kv5)
    for l in range(L):
        at.kv_upload(0, l, 0, kc5, vc5)
    gen = torch.Generator(device=dev).manual_seed(4)
    q = torch.randn(NS5, L, Q_DIM, device=dev, generator=gen)
    k = torch.randn(NS5, L, kv5, device=dev, generator=gen)
    v = torch.randn(NS5, L, kv5, device=dev, generator=gen)
    out = torch.empty(L, Q_DIM, device=dev)
    seq0 = torch.zeros(1, dtype=torch.int32, device=dev)
    posd = (CTX5 + torch.arange(NS5, dtype=torch.int32, device=dev)).contiguous()
    sh = torch.cuda.current_stream(dev).cuda_stream

    def step(s):
        for l in range(L):
            at.decode_batch_dev(l, 1, seq0.data_ptr(), posd[s:s + 1].data_ptr(), CTX5 + NS5 - 1,
                                q[s, l].data_ptr(), k[s, l].data_ptr(), v[s, l].data_ptr(),
                                out[l].data_ptr(), sh)

    step(0)
    torch.cuda.synchronize()
    # the 32 steps captured once and replayed, as in the split version
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        sh_cap = torch.cuda.current_stream(dev).cuda_stream
        for s in range(NS5):
            for l in range(L):
                at.decode_batch_dev(l, 1, seq0.data_ptr(), posd[s:s + 1].data_ptr(),
                                    CTX5 + NS5 - 1, q[s, l].data_ptr(), k[s, l].data_ptr(),
                                    v[s, l].data_ptr(), out[l].data_ptr(), sh_cap)
    graph.replay()
    torch.cuda.synchronize()
    nbytes = sum(L * ((CTX5 + s + 1) * kv5 * 4 + Q_DIM * 8 + kv5 * 12) for s in range(NS5))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    graph.replay()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    del graph
    # decode kernels alone (module events; costs the decode/merge overlap)
    at.profile(True)
    for s in range(NS5):
        step(s)
    torch.cuda.synchronize()
    kern_ms, n_attn, n_all = at.profile_read()
    at.profile(False)
    at.close()
    return {"metric": "long-context decode-attn HBM GB/s (config 5, 1 GPU)",
            "value": nbytes / (ms / 1e3) / 1e9, "unit": "GB/s",
            "pct_peak": 100.0 * nbytes / (ms / 1e3) / 1e9 / peaks["hbm_gbs"],
            "tok_per_s": NS5 / (ms / 1e3), "ms_per_step_16_layers": ms / NS5,
            "attn_kernel_gbs": nbytes / (kern_ms / 1e3) / 1e9, "gpu_launches": n_all,
            "config": {"workload": "config5 16 layers, 32/8 heads, hd 64, theta 5e5, "
                                   "32768 cached + 32 steps, KV N(0,1) seed 4"}}


def run_hd128(args, local, peaks):
    """head_dim 128 (LLaMA-3-8B heads 32/8): batched decode of 32 sequences
    x 2048 cached rows, and the causal prefill of 2048 positions of one layer.
    The decode steps run back to back over two sets of 32 sequences in
    alternation (268 MB of cache each, more than the 126 MB L2), so every
    step reads 268 MB that the step before did not touch, as the headline
    does with its four sets."""
    import torch
    import picolm_b200 as pb
    H8, HK8, HD8, NSEQ, CTX8, NST = 32, 8, 128, 32, 2048, 16
    q_dim, kv_dim = H8 * HD8, HK8 * HD8
    dev = torch.device("cuda", local)
    sh = torch.cuda.current_stream(dev).cuda_stream
    rng = np.random.default_rng(6)
    res = {"config": {"workload": "head_dim 128, heads 32/8 (LLaMA-3-8B), theta 5e5; decode: "
                                  f"{NSEQ} seqs x {CTX8} cached, {NST} steps; prefill: 2048 "
                                  "positions of one layer", "data": "synthetic, seed 6"}}
    # ---- batched decode
    at = pb.Attn(1, H8, HK8, CTX8 + NST, rope_base=500000.0, n_seqs=2 * NSEQ, device=local,
                 head_dim=HD8)
    for s in range(NSEQ):
        kc, vc = make_cache_host(rng, CTX8, kv_dim), make_cache_host(rng, CTX8, kv_dim)
        at.kv_upload(s, 0, 0, kc, vc)
        at.kv_upload(NSEQ + s, 0, 0, kc, vc)  # the second set: same values, other addresses
    gen = torch.Generator(device=dev).manual_seed(6)
    q = torch.randn(NST, NSEQ, q_dim, device=dev, generator=gen)
    k = torch.randn(NST, NSEQ, kv_dim, device=dev, generator=gen)
    v = torch.randn(NST, NSEQ, kv_dim, device=dev, generator=gen)
    out = torch.empty(NSEQ, q_dim, device=dev)
    seqs = [torch.arange(ks * NSEQ, (ks + 1) * NSEQ, dtype=torch.int32, device=dev)
            for ks in range(2)]
    pos = (CTX8 + torch.arange(NST, dtype=torch.int32, device=dev))[:, None].repeat(
        1, NSEQ).contiguous()
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    flush_rd = torch.ones(L2_FLUSH_BYTES // 4, dtype=torch.int32, device=dev)

    def step(j):  # set j % 2 at position index j // 2
        s = j // 2
        at.decode_batch_dev(0, NSEQ, seqs[j % 2].data_ptr(), pos[s].data_ptr(), CTX8 + NST - 1,
                            q[s].data_ptr(), k[s].data_ptr(), v[s].data_ptr(), out.data_ptr(), sh)

    def nbytes(j):
        rows = CTX8 + j // 2 + 1
        return NSEQ * (rows * kv_dim * 4 + q_dim * 8 + kv_dim * 12)

    for j in range(4):
        step(j)
    torch.cuda.synchronize()
    n_steps = 2 * NST
    tot_b = sum(nbytes(j) for j in range(n_steps))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    for j in range(n_steps):
        step(j)
    e1.record()
    torch.cuda.synchronize()
    tot_ms = e0.elapsed_time(e1)
    # the decode kernel in isolation: L2 flushed and the module's events
    # around each launch (set-up exposed, as the headline's isolated figure)
    at.profile(True)
    prof_b = 0
    for j in range(n_steps):
        flush.zero_(); flush_rd.sum(); step(j)
        prof_b += nbytes(j)
    torch.cuda.synchronize()
    kern_ms, _, _ = at.profile_read()
    at.profile(False)
    at.close()
    del flush, flush_rd
    gbs = tot_b / (tot_ms / 1e3) / 1e9
    res["decode"] = {"metric": "decode-attn HBM GB/s (head_dim 128)", "value": gbs,
                     "unit": "GB/s", "pct_peak": 100.0 * gbs / peaks["hbm_gbs"],
                     "ms_per_step": tot_ms / n_steps,
                     "timing": f"{n_steps} steps back to back, two alternating sets of {NSEQ} "
                               "sequences (268 MB of cache each)",
                     "kernel_gbs": prof_b / (kern_ms / 1e3) / 1e9,
                     "kernel_frac": prof_b / (kern_ms / 1e3) / 1e9 / peaks["hbm_gbs"]}
    # ---- prefill of one layer
    S = 2048
    at = pb.Attn(1, H8, HK8, S, rope_base=500000.0, device=local, head_dim=HD8)
    qp = torch.randn(S, q_dim, device=dev, generator=gen).half().float()
    kp = torch.randn(S, kv_dim, device=dev, generator=gen).half().float()
    vp = torch.randn(S, kv_dim, device=dev, generator=gen).half().float()
    op = torch.empty(S, q_dim, device=dev)

    def pf():
        at.prefill_dev(0, 0, 0, S, qp.data_ptr(), kp.data_ptr(), vp.data_ptr(), op.data_ptr(),
                       None, sh)

    for _ in range(3):
        pf()
    torch.cuda.synchronize()
    reps = 5
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        pf()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    # the attention kernel alone (module events; they separate it from the
    # prologue)
    at.profile(True)
    for _ in range(reps):
        pf()
    torch.cuda.synchronize()
    kern_ms, _, _ = at.profile_read()
    at.profile(False)
    at.close()
    flops = 4.0 * H8 * HD8 * S * (S + 1) / 2
    kern_tf = flops * reps / (kern_ms / 1e3) / 1e12
    res["prefill"] = {"metric": "prefill-attn TFLOP/s (head_dim 128, causal FLOPs / call time)",
                      "value": flops / (ms / 1e3) / 1e12, "unit": "TFLOP/s",
                      "ms_per_layer": ms, "attn_kernel_tflops": kern_tf,
                      "attn_kernel_frac": kern_tf / peaks["bf16_tflops"],
                      "traffic": profile_traffic("prefill_attn_kernel_hd128.txt"),
                      "path": "prologue (RoPE + append + q as FP16 high part and residual) "
                              "then the tcgen05 kernel, "
                              "64-row KV tiles"}
    return res


def run_long_ctx_split(args, rank, world, local, peaks):
    """Config 5 split along the KV axis over `world` GPUs: rank r holds a
    contiguous 1/world of the 32768 cached positions (the last rank also the
    appended ones); per layer and step each rank computes its partial
    (m, l, o), pushes it to every rank over NVLink and merges, all in one
    call (pl_attn_decode_p2p_dev through picolm_b200/shard.py).  Timed on
    every rank, max over ranks."""
    import torch
    import picolm_b200 as pb
    from picolm_b200.shard import PART_STRIDE, KVSplitDecoder, P2PShardOps
    L, HK5, CTX5, NS5 = 16, 8, 32768, 32
    kv5 = HK5 * HD
    dev = torch.device("cuda", local)
    # the RoPE tables are indexed by global position, so every rank's
    # context spans all positions; only its shard's rows are filled
    at = pb.Attn(L, H, HK5, CTX5 + NS5, rope_base=500000.0, device=local)
    stream = torch.cuda.current_stream(dev)
    dec = KVSplitDecoder(rank=rank, world=world, n_cached=CTX5,
                         ops=P2PShardOps(at, stream.cuda_stream, rank, world))
    rng = np.random.default_rng(4 + rank)
    # this rank's rows only, one layer's worth uploaded to all 16 layers
    if dec.n_rows:
        kc = make_cache_host(rng, dec.n_rows, kv5)
        vc = make_cache_host(rng, dec.n_rows, kv5)
        for l in range(L):
            at.kv_upload(0, l, 0, kc, vc)
    gen = torch.Generator(device=dev).manual_seed(4)
    q = torch.randn(NS5, L, Q_DIM, device=dev, generator=gen)
    k = torch.randn(NS5, L, kv5, device=dev, generator=gen)
    v = torch.randn(NS5, L, kv5, device=dev, generator=gen)
    out = torch.empty(L, Q_DIM, device=dev)
    part = torch.empty(H * PART_STRIDE, device=dev)
    parts_all = torch.empty(world * H * PART_STRIDE, device=dev)

    def step(s):
        for l in range(L):
            dec.step(l, CTX5 + s, q[s, l], k[s, l], v[s, l], part, parts_all, out[l])

    # the first step appends position CTX5; re-running a step rewrites the
    # same row with the same values, so the warm-up reuses step 0
    step(0)
    torch.cuda.synchronize()
    # all 32 steps x 16 layers captured once and replayed: launched one by
    # one from Python, the host rather than the GPUs would set the pace
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        dec.ops.stream = torch.cuda.current_stream(dev).cuda_stream
        for s in range(NS5):
            step(s)
    dec.ops.stream = stream.cuda_stream
    barrier(world)
    graph.replay()
    torch.cuda.synchronize()
    barrier(world)
    nbytes = sum(L * ((CTX5 + s + 1) * kv5 * 4 + Q_DIM * 8 + kv5 * 12) for s in range(NS5))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    graph.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1), world)
    del graph
    barrier(world)
    at.close()
    return {"metric": f"long-context decode-attn HBM GB/s (config 5, KV split over {world} GPUs)",
            "value": nbytes / (ms / 1e3) / 1e9, "unit": "GB/s",
            "pct_peak_per_gpu": 100.0 * nbytes / (ms / 1e3) / 1e9 / world / peaks["hbm_gbs"],
            "tok_per_s": NS5 / (ms / 1e3), "ms_per_step_16_layers": ms / NS5,
            "timing": "one CUDA graph of all 32 steps, replayed",
            "scaling": "strong", "collective": "per layer the merge grid of every rank's partial "
                                             "(pl_attn_decode_p2p_dev) stores its 32 x 68 FP32 "
                                             "partial into every rank's buffer over NVLink (P2P "
                                             "stores); its last block stamps the epoch, waits for "
                                             "every rank's stamp and merges (LSE)",
            "config": {"workload": "config5 16 layers, 32/8 heads, hd 64, theta 5e5, "
                                   "32768 cached + 32 steps, KV N(0,1) seed 4",
                       "shard": f"{dec.n_rows} cached positions on rank {rank}"}}


def run_long_ctx_heads(args, rank, world, local, peaks):
    """Config 5 split by KV head over `world` GPUs (attention tensor
    parallelism): rank r holds all 32768 cached positions of KV heads
    [8r/world, 8(r+1)/world) and runs their query heads; its output is that
    slice of heads of every layer's attention row, which a row-parallel
    output projection consumes without a gather.  Same data, step structure
    and timing as the KV split (one CUDA graph of the 32 steps x 16 layers,
    max over ranks)."""
    import torch
    import picolm_b200 as pb
    from picolm_b200.shard import head_shard
    L, HK5, CTX5, NS5 = 16, 8, 32768, 32
    kv5 = HK5 * HD
    h0, hq, k0, hk = head_shard(H, HK5, world, rank)
    dev = torch.device("cuda", local)
    at = pb.Attn(L, hq, hk, CTX5 + NS5, rope_base=500000.0, device=local)
    stream = torch.cuda.current_stream(dev)
    rng = np.random.default_rng(4)
    # this rank's KV heads only, one layer's worth uploaded to all 16 layers
    kc = make_cache_host(rng, CTX5, hk * HD)
    vc = make_cache_host(rng, CTX5, hk * HD)
    for l in range(L):
        at.kv_upload(0, l, 0, kc, vc)
    gen = torch.Generator(device=dev).manual_seed(4)
    q = torch.randn(NS5, L, Q_DIM, device=dev, generator=gen)[:, :, h0 * HD:(h0 + hq) * HD]
    k = torch.randn(NS5, L, kv5, device=dev, generator=gen)[:, :, k0 * HD:(k0 + hk) * HD]
    v = torch.randn(NS5, L, kv5, device=dev, generator=gen)[:, :, k0 * HD:(k0 + hk) * HD]
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    out = torch.empty(L, hq * HD, device=dev)
    seq0 = torch.zeros(1, dtype=torch.int32, device=dev)
    posd = (CTX5 + torch.arange(NS5, dtype=torch.int32, device=dev)).contiguous()

    def step(s, sh):
        for l in range(L):
            at.decode_batch_dev(l, 1, seq0.data_ptr(), posd[s:s + 1].data_ptr(), CTX5 + NS5 - 1,
                                q[s, l].data_ptr(), k[s, l].data_ptr(), v[s, l].data_ptr(),
                                out[l].data_ptr(), sh)

    step(0, stream.cuda_stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        sh_cap = torch.cuda.current_stream(dev).cuda_stream
        for s in range(NS5):
            step(s, sh_cap)
    barrier(world)
    graph.replay()
    torch.cuda.synchronize()
    barrier(world)
    nbytes = sum(L * ((CTX5 + s + 1) * kv5 * 4 + Q_DIM * 8 + kv5 * 12) for s in range(NS5))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    graph.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1), world)
    del graph
    barrier(world)
    at.close()
    return {"metric": f"long-context decode-attn HBM GB/s (config 5, split by KV head over "
                      f"{world} GPUs)",
            "value": nbytes / (ms / 1e3) / 1e9, "unit": "GB/s",
            "pct_peak_per_gpu": 100.0 * nbytes / (ms / 1e3) / 1e9 / world / peaks["hbm_gbs"],
            "tok_per_s": NS5 / (ms / 1e3), "ms_per_step_16_layers": ms / NS5,
            "timing": "one CUDA graph of all 32 steps, replayed", "scaling": "strong",
            "collective": "none: each rank's output is its slice of heads",
            "config": {"workload": "config5 16 layers, 32/8 heads, hd 64, theta 5e5, "
                                   "32768 cached + 32 steps, KV N(0,1) seed 4",
                       "shard": f"KV heads {k0}..{k0 + hk - 1} (query heads {h0}..{h0 + hq - 1}) "
                                f"on rank {rank}"}}


def random_q4k(rng, rows: int, n: int) -> np.ndarray:
    """Raw GGUF Q4_K rows (picolm/quant.h:65-72) with dequantised weights of
    mean about 0 and standard deviation about 0.02: random quants and 6-bit
    scales, FP16 d and dmin = 7.5 d (which centres d*sc*q - dmin*mn)."""
    nb = rows * n // 256
    blk = rng.integers(0, 256, (nb, 144), dtype=np.uint8)
    d32 = rng.uniform(0.5, 1.5, nb) * 0.02 / 260
    d = d32.astype(np.float16).view(np.uint8)
    dmin = (d32 * 7.5).astype(np.float16).view(np.uint8)
    blk[:, 0:2] = d.reshape(-1, 2)
    blk[:, 2:4] = dmin.reshape(-1, 2)
    return blk.reshape(rows, -1)


def run_block(args, local, peaks):
    """The whole attention sub-block with its projections (RMSNorm, Q/K/V,
    RoPE, append, attention, output projection, residual) on TinyLlama
    shapes with Q4_K weights (config 2's weight type), one layer:
      * batched decode, 64 sequences x 2048 cached rows (the headline's
        context), L2 flushed before each step, against the attention-only
        step on the same cache;
      * one sequence x 2048 cached rows (a single-stream decode step);
      * causal prefill of 2048 positions, against the attention-only prefill.
    The projections' time is the block's minus the attention's."""
    import torch
    import picolm_b200 as pb
    DIM = 2048
    dev = torch.device("cuda", local)
    sh = torch.cuda.current_stream(dev).cuda_stream
    rng = np.random.default_rng(8)
    gen = torch.Generator(device=dev).manual_seed(8)
    w = [random_q4k(rng, Q_DIM, DIM), random_q4k(rng, KV_DIM, DIM), random_q4k(rng, KV_DIM, DIM),
         random_q4k(rng, DIM, Q_DIM)]
    w_bytes = sum(x.nbytes for x in w)
    norm = (1.0 + 0.1 * rng.standard_normal(DIM)).astype(np.float32)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    flush_rd = torch.ones(L2_FLUSH_BYTES // 4, dtype=torch.int32, device=dev)
    res = {"config": {"workload": "attention sub-block with projections, TinyLlama shapes "
                                  "(dim 2048, 32/4 heads), Q4_K weights, one layer",
                      "weights_bytes": w_bytes, "data": "synthetic, seed 8"}}

    def timed(fn, reps, flush_l2):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        tot = 0.0
        for _ in range(reps):
            if flush_l2:
                flush.zero_(); flush_rd.sum()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(); fn(); e1.record()
            torch.cuda.synchronize()
            tot += e0.elapsed_time(e1)
        return tot / reps

    for n_seq, key in ((SEQS_PER_GPU, "decode_batch64"), (1, "decode_single")):
        at = pb.Attn(1, H, HK, CTX + 8, n_seqs=n_seq, device=local)
        at.set_layer(0, DIM, w[0], pb.PL_GGUF_Q4_K, w[1], pb.PL_GGUF_Q4_K, w[2], pb.PL_GGUF_Q4_K,
                     w[3], pb.PL_GGUF_Q4_K, attn_norm=norm, eps=1e-5)
        for s_ in range(n_seq):
            at.kv_upload(s_, 0, 0, make_cache_host(rng, CTX, KV_DIM),
                         make_cache_host(rng, CTX, KV_DIM))
        x = torch.randn(n_seq, DIM, device=dev, generator=gen)
        q = torch.randn(n_seq, Q_DIM, device=dev, generator=gen)
        k = torch.randn(n_seq, KV_DIM, device=dev, generator=gen)
        v = torch.randn(n_seq, KV_DIM, device=dev, generator=gen)
        out = torch.empty(n_seq, Q_DIM, device=dev)
        seqs = torch.arange(n_seq, dtype=torch.int32, device=dev)
        pos = torch.full((n_seq,), CTX, dtype=torch.int32, device=dev)
        blk = lambda: at.block_decode_dev(0, n_seq, seqs.data_ptr(), pos.data_ptr(), CTX,
                                          x.data_ptr(), sh)
        att = lambda: at.decode_batch_dev(0, n_seq, seqs.data_ptr(), pos.data_ptr(), CTX,
                                          q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                          out.data_ptr(), sh)
        reps = 20 if n_seq > 1 else 200
        ms_blk = timed(blk, reps, flush_l2=True)
        ms_att = timed(att, reps, flush_l2=True)
        # host-buffer call as model.c makes it (registered residual stream)
        xh = np.ascontiguousarray(x.cpu().numpy())
        at.host_register(xh)
        sq, ps = np.arange(n_seq, dtype=np.int32), np.full(n_seq, CTX, np.int32)
        for _ in range(5):
            at.lib.pl_attn_block_decode(0, n_seq, sq, ps, xh.ravel())
        t0 = time.perf_counter()
        for _ in range(reps):
            at.lib.pl_attn_block_decode(0, n_seq, sq, ps, xh.ravel())
        host_ms = (time.perf_counter() - t0) / reps * 1e3
        at.host_unregister(xh)
        at.close()
        kv_b = n_seq * ((CTX + 1) * KV_DIM * 4)
        proj_ms = ms_blk - ms_att
        flops = 2.0 * n_seq * (Q_DIM * DIM + 2 * KV_DIM * DIM + DIM * Q_DIM)
        res[key] = {"sequences": n_seq, "cached_rows": CTX, "ms_block": ms_blk,
                    "ms_attention_only": ms_att, "ms_projections": proj_ms,
                    "projection_weight_gbs": w_bytes / (proj_ms / 1e3) / 1e9,
                    "projection_tflops_fp32": flops / (proj_ms / 1e3) / 1e12,
                    "block_gbs": (kv_b + w_bytes) / (ms_blk / 1e3) / 1e9,
                    "host_call_ms": host_ms,
                    "timing": "CUDA events per step, L2 flushed before each; host call "
                              "wall clock, synchronous"}
    # ---- prefill of 2048 positions
    S = 2048
    at = pb.Attn(1, H, HK, S, device=local)
    at.set_layer(0, DIM, w[0], pb.PL_GGUF_Q4_K, w[1], pb.PL_GGUF_Q4_K, w[2], pb.PL_GGUF_Q4_K,
                 w[3], pb.PL_GGUF_Q4_K, attn_norm=norm, eps=1e-5)
    xp = torch.randn(S, DIM, device=dev, generator=gen)
    qp = torch.randn(S, Q_DIM, device=dev, generator=gen)
    kp = torch.randn(S, KV_DIM, device=dev, generator=gen)
    vp = torch.randn(S, KV_DIM, device=dev, generator=gen)
    op = torch.empty(S, Q_DIM, device=dev)
    ms_blk = timed(lambda: at.block_prefill_dev(0, 0, 0, S, xp.data_ptr(), sh), 5, False)
    ms_att = timed(lambda: at.prefill_dev(0, 0, 0, S, qp.data_ptr(), kp.data_ptr(),
                                          vp.data_ptr(), op.data_ptr(), None, sh), 5, False)
    at.close()
    flops = 2.0 * S * (Q_DIM * DIM + 2 * KV_DIM * DIM + DIM * Q_DIM)
    res["prefill_2048"] = {"ms_block": ms_blk, "ms_attention_only": ms_att,
                           "ms_projections": ms_blk - ms_att,
                           "projection_tflops_fp32": flops / ((ms_blk - ms_att) / 1e3) / 1e12}
    del flush, flush_rd
    return res


def run_decode1(local):
    """Config 1: one TinyLlama decode layer at position 255 (latency)."""
    import picolm_b200 as pb
    rng = np.random.default_rng(0)
    at = pb.Attn(1, H, HK, 256, device=local)
    at.kv_upload(0, 0, 0, make_cache_host(rng, 255, KV_DIM), make_cache_host(rng, 255, KV_DIM))
    q = rng.standard_normal(Q_DIM, dtype=np.float32)
    k = rng.standard_normal(KV_DIM, dtype=np.float32)
    v = rng.standard_normal(KV_DIM, dtype=np.float32)
    out = np.empty(Q_DIM, np.float32)
    raw = at.raw().pl_attn_decode
    ptrs = (q.ctypes.data, k.ctypes.data, v.ctypes.data, out.ctypes.data)
    for _ in range(20):
        assert raw(0, 0, 255, *ptrs) == 0
    n = 500
    t0 = time.perf_counter()
    for _ in range(n):
        raw(0, 0, 255, *ptrs)
    dt = (time.perf_counter() - t0) / n
    at.close()
    return {"metric": "decode layer latency, config 1 (host buffers, synchronous)",
            "us_per_call": dt * 1e6, "bytes_per_call": 281600,
            "api": "pl_attn_decode through a void* ctypes binding, unregistered buffers"}


def run_multi_device(args):
    """One process driving every visible GPU through pl_attn_init_devices (the
    C-ABI fan-out a C caller gets), host buffers:
      seqs  config 4 weak-scaled, 64 sequences x 2048 rows per GPU, one
            pl_attn_decode_batch call a step (PL_SPLIT_SEQS);
      kv    config 5, one 32768-row sequence over 16 layers split along the
            positions (PL_SPLIT_KV), one pl_attn_decode call per layer,
            against the same calls on one GPU."""
    import ctypes as C
    import torch
    import picolm_b200 as pb
    D = args.gpus if args.gpus > 1 else torch.cuda.device_count()
    res = {"devices": D}
    devs = list(range(D))
    # ---- sequences spread over the devices
    n = SEQS_PER_GPU * D
    at = pb.Attn(1, H, HK, CTX + NSTEP, n_seqs=n, devices=devs, split=pb.PL_SPLIT_SEQS)
    rng = np.random.default_rng(3)
    kc = make_cache_host(rng, CTX, KV_DIM)
    for s in range(n):
        at.kv_upload(s, 0, 0, kc, kc)
    q = rng.standard_normal((n, Q_DIM), dtype=np.float32)
    k = rng.standard_normal((n, KV_DIM), dtype=np.float32)
    v = rng.standard_normal((n, KV_DIM), dtype=np.float32)
    out = np.empty((n, Q_DIM), np.float32)
    seqs = np.arange(n, dtype=np.int32)
    for arr in (q, k, v, out):
        at.host_register(arr)
    f = at.raw().pl_attn_decode_batch
    steps = max(args.steps, 20)

    def run(j):
        pos = np.full(n, CTX + j % NSTEP, np.int32)
        rc = f(0, n, seqs.ctypes.data, pos.ctypes.data, q.ctypes.data, k.ctypes.data,
               v.ctypes.data, out.ctypes.data)
        if rc:
            raise pb.PlAttnError(rc, "pl_attn_decode_batch")
        return step_bytes(CTX + j % NSTEP, n)

    for j in range(args.warmup):
        run(j)
    t0 = time.perf_counter()
    nb = sum(run(args.warmup + j) for j in range(steps))
    dt = time.perf_counter() - t0
    for arr in (q, k, v, out):
        at.host_unregister(arr)
    at.close()
    res["seqs"] = {"metric": "config-4 decode through pl_attn_decode_batch, host buffers, "
                             "sequences spread over the devices of one context",
                   "value": nb / dt / 1e9, "unit": "GB/s", "ms_per_step": dt / steps * 1e3,
                   "sequences": n}
    # ---- one long sequence split along the positions, against one GPU
    L, HK5, CTX5 = 16, 8, 32768
    kv5 = HK5 * HD
    base = rng.standard_normal(CTX5 * kv5, dtype=np.float32)
    from oracle import oracle as O
    cache = O.fp32_to_fp16(base).reshape(CTX5, kv5)
    qs = rng.standard_normal((L, Q_DIM), dtype=np.float32)
    ks = rng.standard_normal((L, kv5), dtype=np.float32)
    vs = rng.standard_normal((L, kv5), dtype=np.float32)
    o5 = np.empty(Q_DIM, np.float32)
    for label, dl, split in (("one_gpu", [0], pb.PL_SPLIT_SEQS), ("split", devs, pb.PL_SPLIT_KV)):
        at = pb.Attn(L, H, HK5, CTX5 + 64, rope_base=500000.0, devices=dl, split=split)
        for l in range(L):
            at.kv_upload(0, l, 0, cache, cache)
        d1 = at.raw().pl_attn_decode

        def step5(j):
            p = CTX5 + j
            for l in range(L):
                rc = d1(0, l, p, qs[l].ctypes.data, ks[l].ctypes.data, vs[l].ctypes.data,
                        o5.ctypes.data)
                if rc:
                    raise pb.PlAttnError(rc, "pl_attn_decode")

        step5(0)
        ns = 16
        t0 = time.perf_counter()
        for j in range(1, ns + 1):
            step5(j)
        dt = time.perf_counter() - t0
        nbytes = sum(L * ((CTX5 + j + 1) * kv5 * 4 + Q_DIM * 8 + kv5 * 12) for j in range(1, ns + 1))
        res["kv_" + label] = {"value": nbytes / dt / 1e9, "unit": "GB/s",
                              "ms_per_step_16_layers": dt / ns * 1e3, "devices": len(dl)}
        at.close()
    return res


# ------------------------------------------------------------------ main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["all", "decode", "prefill", "long_ctx", "decode1",
                                           "hd128", "block", "multi_device"],
                    default="all",
                    help="all: headline + configs 1/3/5 + CPU baseline; decode: headline only; "
                         "prefill / long_ctx / decode1 / hd128 / block: that workload alone; "
                         "multi_device: every visible GPU from one process through "
                         "pl_attn_init_devices (run without torchrun)")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    config = {"workload": "config4 batched decode: 64 seqs per GPU x 2048 cached positions, "
                          "TinyLlama heads 32/4, hd 64, 64 decode steps (pos 2048..2111) cycled",
              "seqs_per_gpu": SEQS_PER_GPU, "global_seqs": SEQS_PER_GPU * world,
              "cached_positions": CTX, "parallelism": f"sequence shards x{world}, no collective",
              "l2": "inputs larger than L2, no flush: 4 disjoint sets of 64 sequences "
                    "(4 x 134 MB of cache) in rotation, each step reads the 134 MB that the "
                    "previous 3 steps did not touch (L2 is 126 MB); the timed steps run back "
                    "to back between one barrier + synchronize pair"}
    base = {"metric": "decode-attn HBM GB/s", "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "fp16 KV, fp32 accumulate",
            "data": "synthetic (seeded N(0,1) KV cache and q/k/v)", "config": config}

    if args.impl == "reference":
        if rank != 0:
            return
        r = cpu_decode_sample(steps=args.steps, warmup=args.warmup)
        line = dict(base)
        line.update({"impl": "reference", "value": r["value"],
                     "ms_per_step": r["s_per_step"] * 1e3, "steps": r["steps"],
                     "warmup": args.warmup,
                     "cpu_baseline": {k: r[k] for k in ("value", "unit", "cores", "kind",
                                                        "sample")},
                     "e2e": {"value": r["value"], "unit": "GB/s", "h2d_bytes_per_step": 0,
                             "d2h_bytes_per_step": 0}})
        print(json.dumps(line), flush=True)
        return

    rank, world, local = dist_setup()
    from picolm_b200 import build
    if rank == 0:
        build.build()
    barrier(world)
    peaks = load_peaks()
    if args.workload == "long_ctx" and world > 1:
        r = run_long_ctx_split(args, rank, world, local, peaks)
        r["by_kv_head"] = run_long_ctx_heads(args, rank, world, local, peaks)
        if rank == 0:
            print(json.dumps(r), flush=True)
        import torch.distributed as dist
        dist.destroy_process_group()
        return
    if args.workload == "multi_device":
        # one process drives every GPU itself (no torchrun)
        if rank == 0:
            print(json.dumps(run_multi_device(args)), flush=True)
        return
    if args.workload in ("prefill", "long_ctx", "decode1", "hd128", "block"):
        if rank == 0:
            fn = {"prefill": lambda: run_prefill(args, local, peaks),
                  "long_ctx": lambda: run_long_ctx(args, local, peaks),
                  "decode1": lambda: run_decode1(local),
                  "hd128": lambda: run_hd128(args, local, peaks),
                  "block": lambda: run_block(args, local, peaks)}[args.workload]
            print(json.dumps(fn()), flush=True)
        return
    res = run_batched_decode(args, rank, world, local, peaks)
    line = dict(base)
    line.update({"impl": "ours", "value": res["value"], "ms_per_step": res["ms_per_step"],
                 "tok_per_s": res["tok_per_s"], "pct_peak": res["pct_peak"],
                 "roofline": res["roofline"], "e2e": res["e2e"],
                 "gpu_launches": res["gpu_launches"], "clocks": res["clocks"],
                 "rank_ms_per_step": res["rank_ms_per_step"]})
    if world > 1 and args.workload == "all":
        line["long_ctx_split"] = run_long_ctx_split(args, rank, world, local, peaks)
        line["long_ctx_heads"] = run_long_ctx_heads(args, rank, world, local, peaks)
    if world == 1 and args.workload == "all":
        line["prefill"] = run_prefill(args, local, peaks)
        line["long_ctx"] = run_long_ctx(args, local, peaks)
        line["decode1"] = run_decode1(local)
        line["hd128"] = run_hd128(args, local, peaks)
        line["block"] = run_block(args, local, peaks)
        cb = cpu_decode_sample(max_seconds=15.0)
        line["cpu_baseline"] = {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")}
        # the reference CPU path beside the other configs' GPU numbers
        line["decode1"]["cpu_baseline"] = cpu_config1_sample()
        line["prefill"]["cpu_baseline"] = cpu_prefill_sample()
        line["long_ctx"]["cpu_baseline"] = cpu_long_ctx_sample()
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
