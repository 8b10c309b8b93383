#!/usr/bin/env python
"""Threefry 32-bit words/s on B200: random_bits(random_key(123), (2^34,)) uint32.

The workload is the bulk-bits request (64 GiB of uint32, jax_threefry_partitionable
layout, 32-bit mode), split by contiguous counter range over the N GPUs of one node:
rank r writes elements [r 2^34/N, (r+1) 2^34/N) into its own HBM with no
communication.  A step is one pass of that request; value = 2^34 words / the max over
ranks of the device time per step.

    python bench.py [--gpus N --steps K --warmup W]      # our kernels
    python bench.py --impl reference                      # the CPU implementation

For N > 1 launch one process per GPU with torch.distributed.run.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

TOTAL = 1 << 34          # words per step (the 2^34-word request)
SEED = 123
METRIC = "threefry 32-bit words/s (device-timed) at 1/2/4/8 B200; % of INT-pipe roofline"
OPS_PER_BLOCK = 100      # the metric's integer-op count per 64-bit cipher block
PEAKS = os.path.join(ROOT, "MEASURED_PEAKS.json")
# HBM copy bandwidth of this pool's B200s measured earlier, for when the per-pod
# MEASURED_PEAKS.json is absent
HBM_FALLBACK_GBS = 6650.0


def hbm_peak_gbs():
    """(peak GB/s, where it comes from): MEASURED_PEAKS.json's hbm_gbs, else the fallback."""
    try:
        return float(json.load(open(PEAKS))["hbm_gbs"]), "MEASURED_PEAKS.json hbm_gbs (of measured)"
    except (OSError, ValueError, KeyError, TypeError):
        return HBM_FALLBACK_GBS, "fallback 6650 GB/s (MEASURED_PEAKS.json absent; of fallback)"
TRAFFIC = os.path.join(ROOT, "profiles", "traffic.json")


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def config_block(args, world, e2e_words=None):
    c = {"workload": "random_bits(random_key(123L), shape=(2^34,)) uint32, "
                     "jax_threefry_partitionable, x32",
         "request_words": TOTAL, "per_gpu_words": TOTAL // world, "sharding": "contiguous counter range",
         "parallelism": f"counter-range x{world}", "l2": "outputs larger than L2 (no flush needed)"}
    if e2e_words:
        c["e2e_words_per_gpu"] = e2e_words
    return c


# ---- clocks during the timed region ------------------------------------------------------------

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index):
        self.dev = device_index
        self.proc = None
        self.path = f"/tmp/jxr_clocks_{os.getpid()}.csv"

    def start(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.dev)], stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.f.close()
        rows = []
        for ln in open(self.path):
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None
        mhz = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(mhz) if mhz else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons, "samples": len(rows)}


# ---- the CPU implementation (oracle port, all host threads) -------------------------------------

def cpu_words_per_s(min_seconds=3.0, sample=1 << 27):
    """Bulk partitionable uint32 bits of the same request on the host cores: the first
    `sample` words of the 2^34-word request, repeated until min_seconds have passed."""
    import numpy as np
    from oracle import oracle as orc
    key = orc.seed(SEED)
    threads = os.cpu_count() or 1
    orc.set_threads(threads)
    out = np.empty(sample, dtype=np.uint32)
    lib = orc.lib()
    import ctypes
    k = (ctypes.c_uint32 * 2)(int(key[0]), int(key[1]))
    lib.orc_random_bits(k, 32, TOTAL, 1, 0, sample, out.ctypes.data_as(ctypes.c_void_p))  # warm
    reps, t0 = 0, time.perf_counter()
    while True:
        lib.orc_random_bits(k, 32, TOTAL, 1, reps * sample % TOTAL, sample,
                            out.ctypes.data_as(ctypes.c_void_p))
        reps += 1
        dt = time.perf_counter() - t0
        if dt >= min_seconds:
            break
    return reps * sample / dt, threads, f"first {reps} x 2^{sample.bit_length() - 1} words of the request"


def run_reference(args):
    rank = int(os.environ.get("RANK", 0))
    if rank != 0:
        return 0
    import numpy as np  # noqa: F401
    from oracle import oracle as orc
    orc.build()
    vals = []
    for _ in range(args.warmup):
        cpu_words_per_s(min_seconds=0.5)
    sample_desc, threads = "", 1
    for _ in range(args.steps):
        v, threads, sample_desc = cpu_words_per_s(min_seconds=1.0)
        vals.append(v)
    value = statistics.median(vals)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "words/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": TOTAL / value * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "u32", "data": "synthetic (seeds only)",
        "config": config_block(args, args.gpus),
        "cpu_baseline": {"value": value, "unit": "words/s", "cores": threads, "kind": "port",
                         "sample": sample_desc + " per step; the reference (R + XLA CPU PJRT "
                                   "plugin) cannot run here, so its C restatement runs, "
                                   "OpenMP over all host threads"},
        "e2e": {"value": value, "unit": "words/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    emit(line)
    return 0


# ---- our kernels ---------------------------------------------------------------------------------

def probe_peak(torch, nat, dev, iters=2000):
    """Blocks/s of the register-resident cipher (the integer-pipe ceiling), best of 3."""
    import ctypes
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    best = 0.0
    for cps in (4, 8):
        sink = torch.empty(sms * cps * 256, dtype=torch.int32, device=dev)
        blocks = ctypes.c_uint64(0)
        st = torch.cuda.current_stream().cuda_stream
        nat.call("jxr_probe_cipher", 10, cps, sink.data_ptr(), ctypes.byref(blocks), st)
        for _ in range(3):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            nat.call("jxr_probe_cipher", iters, cps, sink.data_ptr(), ctypes.byref(blocks), st)
            e1.record()
            e1.synchronize()
            best = max(best, blocks.value / (e0.elapsed_time(e1) * 1e-3))
    return best


# ---- the other named workloads C1-C3, C5 and the derived samplers (N = 1, one line each) ----

WORKLOADS = {
    "c1": "random_bits(random_key(0L), shape=(2^20,)) uint32, partitionable, x32",
    "c2": "random_normal(random_key(42L), shape=(8192, 8192)) float32, partitionable",
    "c2o": "random_normal(random_key(42L), shape=(8192, 8192)) float32, original layout",
    "c3": "vmap(function(k) random_uniform(k, 1024, minval=-2, maxval=3))(random_split(random_key(7L), 65536)) float32",
    "c5": "x64: random_normal(random_fold_in(random_key(2024L), 17L), (16384, 16384)) float64 and "
          "random_bernoulli(same key, 0.3, same shape), one fused pass",
    "exp": "random_exponential(random_key(7L), (8192, 8192)) float32",
    "gumbel": "random_gumbel(random_key(7L), (8192, 8192)) float32, mode low",
    "logistic": "random_logistic(random_key(7L), (8192, 8192)) float32",
    "truncnorm": "random_truncated_normal(random_key(7L), -1, 2, (8192, 8192)) float32",
    "randint": "random_randint(random_key(7L), (8192, 8192), 0L, 1000L) int32 "
               "(split, then both 32-bit draws and the combine in one kernel)",
    "perm": "random_permutation(random_key(7L), 2^26) int32: 3 shuffle rounds, each 2^26 "
            "32-bit sort keys, 2 stable radix passes over their top 16 bits and the span sort "
            "of every run of equal top bits in shared memory",
    "rbg": "random_bits(random_key(0L, impl = \"rbg\"), 2^30) uint32: XLA RngBitGenerator "
           "(Philox4x32-10), 4 words per block",
}

# Kernels of this library one call launches (1 unless listed): randint = split and the
# fused draws + combine; perm = per round the key split, the sort keys with the first
# pass's counts, the second pass's counts, 2 x (scan, scatter) and the span sort (round 0's
# first scatter takes the positions as values).
LAUNCHES_PER_CALL = {"randint": 2, "perm": 3 * 8}

# Algorithmic HBM bytes per element of one shuffle round: the 32-bit sort keys written
# once (their first-pass counts taken on the way); per radix pass the (key, position) pair
# read and written, the second pass also reading the keys for its counts; the span sort
# reads the pair and writes the position.
PERM_BYTES_PER_ROUND = 4 + 16 + (4 + 16) + 8 + 4
# three rounds; round 0's first pass takes the positions as values (4 B not read)
PERM_BYTES_PER_CALL = 3 * PERM_BYTES_PER_ROUND - 4

_SAMPLER_WORKLOADS = {"exp": "exponential", "gumbel": "gumbel", "logistic": "logistic"}


def workload_cpu_baseline(c, min_seconds=2.0):
    """The same workload's first outputs computed by the oracle port on all host threads,
    repeated for about min_seconds: 32-bit output words per second."""
    import ctypes

    import numpy as np
    from oracle import oracle as orc
    lib = orc.lib()
    threads = os.cpu_count() or 1
    orc.set_threads(threads)
    if c in _SAMPLER_WORKLOADS or c in ("truncnorm", "randint"):
        return sampler_cpu_baseline(c, min_seconds)
    if c == "rbg":  # the C restatement of the Philox stream, 2^24 words
        n = 1 << 24
        out = np.empty(n, dtype=np.uint32)
        q = orc._key4([0, 0, 0, 0])
        lib.orc_rbg_bits(q, 32, 1 << 30, 0, n, out.ctypes.data_as(ctypes.c_void_p))
        reps, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < min_seconds:
            lib.orc_rbg_bits(q, 32, 1 << 30, 0, n, out.ctypes.data_as(ctypes.c_void_p))
            reps += 1
        dt = time.perf_counter() - t0
        return {"value": reps * n / dt, "unit": "words/s", "cores": threads, "kind": "port",
                "sample": f"first 2^24 words, {reps} times (C restatement, OpenMP)"}
    if c == "perm":  # the restatement (C bits, numpy stable argsort) on 2^22 elements
        n = 1 << 22
        orc.set_threads(threads)
        orc.permutation(orc.seed(7), n)
        reps, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < min_seconds:
            orc.permutation(orc.seed(7), n)
            reps += 1
        dt = time.perf_counter() - t0
        return {"value": reps * n / dt, "unit": "words/s", "cores": threads, "kind": "port",
                "sample": f"random_permutation of 2^22 (3 rounds, as 2^26), {reps} times "
                          "(C bits on all threads, numpy stable argsort on one)"}
    if c == "c1":
        key, n, words_per, fn = orc.seed(0), 1 << 20, 1, "bits"
    elif c in ("c2", "c2o"):
        key, n, words_per, fn = orc.seed(42), 1 << 22, 1, "normal32"
    elif c == "c3":
        key, n, words_per, fn = orc.split(orc.seed(7), 1, True)[0], 1 << 22, 1, "uniform32"
    else:
        key, n, words_per, fn = orc.fold_in(orc.seed(2024, True), 17), 1 << 21, 2, "normal64"
    size = {"c1": 1 << 20, "c2": 1 << 26, "c2o": 1 << 26, "c3": 1024, "c5": 1 << 28}[c]
    part = int(c != "c2o")
    k = (ctypes.c_uint32 * 2)(int(key[0]), int(key[1]))
    out = np.empty(n, dtype=np.float64 if fn == "normal64" else np.uint32)
    optr = out.ctypes.data_as(ctypes.c_void_p)

    def once():
        if fn == "bits":
            lib.orc_random_bits(k, 32, size, part, 0, n, optr)
        elif fn == "normal32":
            lib.orc_normal(k, orc.F32, size, part, 1, 0, n, optr)
        elif fn == "uniform32":  # the same per-output work as 4096 rows of 1024, one key
            lib.orc_uniform(k, orc.F32, n, 1, -2.0, 3.0, 1, 0, n, optr)
        else:
            lib.orc_normal(k, orc.F64, size, part, 1, 0, n, optr)
    once()
    reps, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < min_seconds:
        once()
        reps += 1
    dt = time.perf_counter() - t0
    return {"value": reps * n * words_per / dt, "unit": "words/s", "cores": threads, "kind": "port",
            "sample": f"first {n} outputs of the workload, {reps} times (C restatement, OpenMP)"}


def sampler_cpu_baseline(c, min_seconds=2.0):
    """The derived-sampler workloads' first 2^22 outputs by the oracle port on all host
    threads (randint: the two bit draws in C, the modular combine in numpy)."""
    import ctypes

    import numpy as np
    from oracle import oracle as orc
    lib = orc.lib()
    threads = os.cpu_count() or 1
    orc.set_threads(threads)
    n, size = 1 << 22, 1 << 26
    key = orc.seed(7)
    k = (ctypes.c_uint32 * 2)(int(key[0]), int(key[1]))
    out = np.empty(n, dtype=np.float32)
    optr = out.ctypes.data_as(ctypes.c_void_p)

    def once():
        if c in _SAMPLER_WORKLOADS:
            lib.orc_sample(k, orc.SAMPLE_KIND[_SAMPLER_WORKLOADS[c]], orc.F32, size, 1, 0, n, optr)
        elif c == "truncnorm":
            lib.orc_truncated_normal(k, orc.F32, size, 1, -1.0, 2.0, 1, 0, n, optr)
        else:
            ks = orc.split(key, 2, True)
            hi = orc.random_bits(ks[0], 32, size, True, 0, n).astype(np.uint64)
            lo = orc.random_bits(ks[1], 32, size, True, 0, n).astype(np.uint64)
            span = np.uint64(1000)
            mult = np.uint64((1 << 32) % 1000)
            off = ((hi % span) * mult % (np.uint64(1) << np.uint64(32)) + lo % span) % span
            out.view(np.int32)[:] = off.astype(np.int32)
    once()
    reps, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < min_seconds:
        once()
        reps += 1
    dt = time.perf_counter() - t0
    return {"value": reps * n / dt, "unit": "words/s", "cores": threads, "kind": "port",
            "sample": f"first {n} outputs of the workload, {reps} times (C restatement, OpenMP"
                      + (", numpy combine)" if c == "randint" else ")")}


def run_workload(args):
    """One JSON line for a secondary workload: device time per call of the public API,
    32-bit words of output per second, and the cipher-block rate against the probe."""
    import torch

    import jaxr_b200 as jr
    from jaxr_b200 import _native as nat
    from jaxr_b200 import build as jb
    jb.build()
    nat.lib()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    c = args.config
    flags = {"x64": c == "c5", "part": c != "c2o"}
    old = (jr.enable_x64(flags["x64"]), jr.jax_config_update("jax_threefry_partitionable", flags["part"]))
    if c == "c1":
        key = jr.random_key(0)
        step = lambda: jr.random_bits(key, (1 << 20,))
        words, blocks, out_bytes, dt = 1 << 20, 1 << 20, 4 << 20, "u32"
    elif c in ("c2", "c2o"):
        key = jr.random_key(42)
        step = lambda: jr.random_normal(key, (8192, 8192))
        words, out_bytes, dt = 1 << 26, 4 << 26, "f32"
        blocks = words if c == "c2" else words // 2
    elif c == "c3":
        keys = jr.random_split(jr.random_key(7), 65536)
        f = jr.vmap(lambda k: jr.random_uniform(k, (1024,), minval=-2, maxval=3))
        step = lambda: f(keys)
        words, blocks, out_bytes, dt = 1 << 26, 1 << 26, 4 << 26, "f32"
    elif c == "c5":
        key = jr.random_fold_in(jr.random_key(2024), 17)
        step = lambda: jr.random_normal_bernoulli(key, 0.3, (16384, 16384))
        words, blocks, out_bytes, dt = 1 << 29, 1 << 28, 9 << 28, "f64"
    elif c in _SAMPLER_WORKLOADS or c == "truncnorm":
        key = jr.random_key(7)
        if c == "truncnorm":
            step = lambda: jr.random_truncated_normal(key, -1, 2, (8192, 8192))
        else:
            fn = getattr(jr, "random_" + _SAMPLER_WORKLOADS[c])
            step = lambda: fn(key, (8192, 8192))
        words, blocks, out_bytes, dt = 1 << 26, 1 << 26, 4 << 26, "f32"
    elif c == "randint":
        key = jr.random_key(7)
        step = lambda: jr.random_randint(key, (8192, 8192), 0, 1000)
        # two cipher blocks per output (one per split key half), the int32 result written
        words, blocks, out_bytes, dt = 1 << 26, 1 << 27, 4 << 26, "int32"
    elif c == "rbg":
        key = jr.random_key(0, impl="rbg")
        step = lambda: jr.random_bits(key, (1 << 30,))
        # a store-bound stream: 2^28 Philox blocks, 4 GiB written
        words, blocks, out_bytes, dt = 1 << 30, 1 << 28, 4 << 30, "u32"
    elif c == "perm":
        key = jr.random_key(7)
        step = lambda: jr.random_permutation(key, 1 << 26)
        # 3 rounds: 2^26 cipher blocks each, PERM_BYTES_PER_CALL bytes per element in all
        words, blocks, out_bytes, dt = 1 << 26, 3 << 26, PERM_BYTES_PER_CALL << 26, "int32"
    else:
        raise SystemExit(f"unknown config {c}")
    small = out_bytes < (1 << 30)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev) if small else None
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    sampler = ClockSampler(0)
    sampler.start()
    time.sleep(0.25)
    total = 0.0
    if small:  # outputs fit in L2: flush it before every timed call
        for _ in range(args.steps):
            flush.fill_(1)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            r = step()
            e1.record()
            e1.synchronize()
            total += e0.elapsed_time(e1)
            del r
    else:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            step()
        e1.record()
        e1.synchronize()
        total = e0.elapsed_time(e1)
    clocks = sampler.stop()
    ms = total / args.steps
    peak_blocks = probe_peak(torch, nat, dev)
    hbm_peak, hbm_src = hbm_peak_gbs()
    bps = blocks / (ms * 1e-3)
    gbs = out_bytes / (ms * 1e-3) / 1e9
    hbm = {"achieved": gbs, "peak": hbm_peak, "unit": "GB/s", "frac": gbs / hbm_peak,
           "peak_source": hbm_src}
    if c == "perm":  # a sort: memory-bound, the cipher is 3 blocks per element
        roofline = dict(hbm, bound="hbm", bytes_per_element=PERM_BYTES_PER_CALL,
                        int_frac=bps / peak_blocks)
    elif c == "rbg":  # Philox: ~40 multiplies per 4 words, below the store bandwidth
        roofline = dict(hbm, bound="hbm", bytes_per_element=4)
    else:
        roofline = {"bound": "int", "unit": "Tops/s", "achieved": bps * OPS_PER_BLOCK / 1e12,
                    "peak": peak_blocks * OPS_PER_BLOCK / 1e12, "frac": bps / peak_blocks,
                    "ops_per_block": OPS_PER_BLOCK, "hbm": hbm}
    library = None
    if c == "perm":  # NVIDIA's radix sort on the same pairs: CUB through torch.sort(stable)
        keys = jr.random_bits(jr.random_key(7), (1 << 26,)).view(torch.int32)
        for _ in range(args.warmup):
            torch.sort(keys, stable=True)
        torch.cuda.synchronize()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record()
        for _ in range(args.steps):
            torch.sort(keys, stable=True)
        g1.record()
        g1.synchronize()
        cub_ms = g0.elapsed_time(g1) / args.steps
        library = {"what": "torch.sort(2^26 int32 keys, stable=True): CUB's radix sort of the "
                           "same (32-bit key, position) pairs, one sort", "ms": cub_ms,
                   "per_round_ms_here": ms / 3, "round_vs_library": ms / 3 / cub_ms}
        del keys
    cpu = None if args.no_cpu_baseline else workload_cpu_baseline(c)
    line = {
        "metric": "threefry 32-bit words/s (device-timed), secondary workload", "value": words / (ms * 1e-3),
        "unit": "words/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": None, "vs_baseline": None,
        "dtype": dt, "data": "synthetic (seeds only)",
        "config": {"workload": WORKLOADS[c], "name": c, "output_bytes": out_bytes,
                   "cipher_blocks": blocks,
                   "l2": "flushed (256 MiB write) before every timed call" if small else
                         "outputs larger than L2"},
        "roofline": roofline,
        "gpu_launches": args.steps * LAUNCHES_PER_CALL.get(c, 1), "clocks": clocks,
        "cpu_baseline": cpu,
    }
    if library is not None:
        line["library_baseline"] = library
    jr.enable_x64(old[0])
    jr.jax_config_update("jax_threefry_partitionable", old[1])
    emit(line)
    return 0


def bind_to_gpu_cpus(torch, dev_index):
    """Restrict this process to the CPUs NVML reports as local to the GPU (NUMA), so that
    pinned host buffers are allocated next to it; returns the previous CPU set, or None
    when NVML cannot say.  Only this process's affinity changes."""
    try:
        import pynvml
        p = torch.cuda.get_device_properties(dev_index)
        bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
        pynvml.nvmlInit()
        try:
            h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            words = ((os.cpu_count() or 64) + 63) // 64
            mask = pynvml.nvmlDeviceGetCpuAffinity(h, words)
        finally:
            pynvml.nvmlShutdown()
        cpus = {64 * w + b for w, m in enumerate(mask) for b in range(64) if (int(m) >> b) & 1}
        old = os.sched_getaffinity(0)
        cpus &= old
        if cpus and cpus != old:
            os.sched_setaffinity(0, cpus)
            return old
    except Exception as e:  # noqa: BLE001 - affinity is an optimisation only
        log(f"note: no NUMA binding ({type(e).__name__}: {e})")
    return None


def run_ours(args):
    import torch
    import torch.distributed as dist

    import jaxr_b200 as jr
    from jaxr_b200 import _native as nat
    from jaxr_b200 import build as jb
    from jaxr_b200.shard import random_bits_shard, random_bits_to_host, shard_range

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        log(f"note: --gpus {args.gpus} but WORLD_SIZE={world}; using WORLD_SIZE")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    all_cpus = bind_to_gpu_cpus(torch, local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=dev)
    jb.build()
    nat.lib()

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    key = jr.random_key(SEED)
    lo, hi = shard_range(TOTAL, rank, world)
    out = torch.empty(hi - lo, dtype=torch.uint32, device=dev)

    def step():
        random_bits_shard(key, (TOTAL,), rank, world, out=out)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier()
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.25)
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop()
    ms = e0.elapsed_time(e1) / args.steps
    ms_max = max_over_ranks(ms)
    value = TOTAL / (ms_max * 1e-3)
    per_rank = None
    if world > 1:  # every rank's step time and clocks, for the line (rank 0 prints)
        per_rank = [None] * world
        dist.all_gather_object(per_rank, {"rank": rank, "ms_per_step": ms, "clocks": clocks})

    # roofline of the kernel on this GPU: cipher blocks/s against the register-resident
    # cipher's ceiling, and output bytes/s against measured HBM bandwidth
    peak_blocks = probe_peak(torch, nat, dev)
    my_blocks = (hi - lo) / (ms * 1e-3)
    hbm_peak, hbm_src = hbm_peak_gbs()
    traffic, evidence = None, None
    try:
        tr = json.load(open(TRAFFIC))["bits_u32"]
        traffic = tr["dram_bytes_per_word"] * (hi - lo)
        evidence = tr.get("ncu")
    except (OSError, ValueError, KeyError):
        pass
    roofline = {
        "bound": "int", "unit": "Tops/s",
        "achieved": my_blocks * OPS_PER_BLOCK / 1e12,
        "peak": peak_blocks * OPS_PER_BLOCK / 1e12,
        "frac": my_blocks / peak_blocks,
        "ops_per_block": OPS_PER_BLOCK,
        "peak_source": "measured: jxr_probe_cipher (threefry20 in registers, no memory), this GPU",
        "traffic": traffic,
        # why frac is a true fraction of the integer pipes, independent of the probe: the
        # kernel's own ncu counters (ALU pipe, issue slots, instructions per word)
        "ncu_evidence": evidence,
        "hbm": {"achieved": my_blocks * 4 / 1e9, "peak": hbm_peak, "unit": "GB/s",
                "frac": my_blocks * 4 / 1e9 / hbm_peak, "peak_source": hbm_src},
    }
    # the nominal ceiling too: every SM lane issuing one 32-bit integer op per cycle at the
    # SM clock sampled during the timed region, 100 ops per block
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    mhz = (clocks or {}).get("sm_mhz") or 1965.0
    nominal = sms * 128 * mhz * 1e6 / 1e12
    roofline["nominal"] = {"peak": nominal, "unit": "Tops/s",
                           "frac": my_blocks * OPS_PER_BLOCK / 1e12 / nominal,
                           "source": f"{sms} SMs x 128 lanes x {mhz:.0f} MHz (one integer op "
                                     "per lane per cycle); the cipher issues ~77 instructions "
                                     "per block, part of them on the FMA pipe, so this can "
                                     "exceed 1"}

    # the whole request on rank 0 (timed separately from generation): rank r's kernel
    # storing its slab straight into rank 0's HBM over NVLink, and, for comparison,
    # generating slabs locally then assembling them with NCCL point-to-point
    gather = None
    if world > 1 and not args.no_gather:
        from jaxr_b200.shard import close_peer_mappings, gather_to, random_bits_gathered

        def timed(fn, reps=3):
            fn()
            best = None
            for _ in range(reps):
                barrier()
                torch.cuda.synchronize()
                g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                g0.record()
                r = fn()
                g1.record()
                g1.synchronize()
                del r
                t = max_over_ranks(g0.elapsed_time(g1))
                best = t if best is None else min(best, t)
            return best

        nccl_ms = timed(lambda: gather_to(random_bits_shard(key, (TOTAL,), rank, world, out=out), 0))
        torch.cuda.empty_cache()
        whole = torch.empty(TOTAL, dtype=torch.uint32, device=dev) if rank == 0 else None
        direct_ms = timed(lambda: random_bits_gathered(key, (TOTAL,), root=0, out=whole))
        close_peer_mappings()
        del whole
        torch.cuda.empty_cache()
        into_root = TOTAL * 4 * (world - 1) / world
        gather = {"root": 0, "bytes": TOTAL * 4, "unit": "ms",
                  "direct_ms": direct_ms, "nccl_ms": nccl_ms,
                  "direct_nvlink_GBps_into_root": into_root / (direct_ms * 1e-3) / 1e9,
                  "note": "whole 2^34-word request assembled on rank 0, max over ranks: direct = "
                          "every rank's kernel stores its slab into rank 0's buffer through a "
                          "CUDA IPC peer mapping (random_bits_gathered); nccl = each rank "
                          "generates its slab locally, then NCCL point-to-point to rank 0"}

    # end to end through the public API with a host buffer: key in, bits out to pinned
    # host memory, chunked generation overlapped with the copies
    e2e = None
    e2e_words = None
    if not args.no_e2e:
        e2e_words = min(hi - lo, args.e2e_words)
        host = torch.empty(e2e_words, dtype=torch.uint32, pin_memory=True)
        random_bits_to_host(key, (e2e_words,), out=host)  # warm
        barrier()
        t0 = time.perf_counter()
        for _ in range(args.e2e_steps):
            random_bits_to_host(key, (e2e_words,), out=host)
        dt = max_over_ranks((time.perf_counter() - t0) / args.e2e_steps)
        e2e = {"value": e2e_words * world / dt, "unit": "words/s", "h2d_bytes_per_step": 8,
               "d2h_bytes_per_step": e2e_words * 4 * world,
               "note": "random_bits_to_host of 2^%d words per GPU per step into pinned host "
                       "memory; the key goes host->device and every word device->host inside "
                       "the timed region" % (e2e_words.bit_length() - 1)}
        del host

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        if all_cpus:  # the CPU baseline gets every host core back
            os.sched_setaffinity(0, all_cpus)
        v, threads, sample = cpu_words_per_s()
        cpu = {"value": v, "unit": "words/s", "cores": threads, "kind": "port",
               "sample": sample + " (C restatement of the reference, OpenMP)"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "words/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "u32",
            "data": "synthetic (seeds only; the request is generated from random_key(123))",
            "config": config_block(args, world, e2e_words),
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e,
            "gpu_launches": args.steps, "clocks": clocks,
        }
        if gather is not None:
            line["gather"] = gather
        if per_rank is not None:
            line["nranks"] = world
            line["per_rank"] = per_rank
            # the run's clocks: every rank's sampled median, and every reason any rank saw
            line["clocks"] = dict(clocks or {}, sm_mhz_per_rank=[(r["clocks"] or {}).get("sm_mhz")
                                                                 for r in per_rank],
                                  reasons=sorted({x for r in per_rank
                                                  for x in ((r["clocks"] or {}).get("reasons") or [])}))
        emit(line)
    del out
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


_JSON_OUT = None


def keep_stdout_for_json():
    """Route file descriptor 1 to stderr for the rest of the process (library banners,
    e.g. NCCL's version line, land there) and keep the original stdout for the JSON
    result lines alone."""
    global _JSON_OUT
    if _JSON_OUT is None:
        sys.stdout.flush()
        fd = os.dup(1)
        os.dup2(2, 1)
        _JSON_OUT = os.fdopen(fd, "w")


def emit(line):
    keep_stdout_for_json()
    _JSON_OUT.write(json.dumps(line) + "\n")
    _JSON_OUT.flush()


def main():
    keep_stdout_for_json()
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", default="c4",
                    help="c4 = the 2^34-word bits request (the benchmark); c1, c2, c2o, c3, c5 = "
                         "the other workloads, one GPU, one JSON line each; exp, gumbel, "
                         "logistic, truncnorm, randint, perm, rbg = the derived samplers, the "
                         "permutation and rbg bits; 'all' = every secondary workload; "
                         "'samplers' = those last seven")
    ap.add_argument("--words-log2", type=int, default=34,
                    help="request size 2^k words (34 = the benchmark; smaller only for profiling)")
    ap.add_argument("--e2e-words", type=int, default=1 << 30)
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-gather", action="store_true",
                    help="N > 1: skip timing the whole request assembled on rank 0")
    args = ap.parse_args()
    if args.warmup < 3:
        log("note: warmup raised to 3")
        args.warmup = 3
    global TOTAL
    TOTAL = 1 << args.words_log2
    if args.impl == "reference":
        return run_reference(args)
    if args.config in ("all", "samplers"):
        rc = 0
        names = (["c1", "c2", "c2o", "c3", "c5"] if args.config == "all" else []) + list(
            WORKLOADS)[5:]
        for c in names:
            args.config = c
            rc |= run_workload(args)
        return rc
    if args.config != "c4":
        return run_workload(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
