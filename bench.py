#!/usr/bin/env python3
"""Benchmark: MXFP6 GEMM TFLOPS on B200 (BASELINE metric), one JSON line on rank 0.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config cfg2]

Workload (a "step" = one D = A·B call over one batch of synthetic operands):
  N=1   BASELINE config 2: M=N=K=8192, FP16 out, E2M3 codes uniform over all 64 codes, E8M0
        exponents uniform in [118, 136] (seeded; no dataset).
  N>1   the same per-GPU shape, N-sharded (column-parallel): the job is D[8192, 8192*N] =
        A[8192, 8192] · B[8192, 8192*N] with A replicated and B / D split by columns, so per-GPU
        work is fixed (weak scaling) and no collective sits on the GEMM path.
Other configs (--config cfg1..cfg5) run the same harness on BASELINE's other shapes.

Every line also carries
  "strong"      BASELINE config 5 (the FFN up-projection 4096 x 28672 x 8192, BF16 out) with B and
                D split column-parallel over the N ranks: total and per-GPU TFLOPS, the same
                GEMM unsplit on one GPU, the efficiency against it, whether the shard results
                equal the unsplit D bit for bit, and the optional D all-gather (NCCL, and the
                fused epilogue gather over NVLink peer stores) at N>1;
  "per_config"  (N=1) device-timed TFLOPS, route and roofline fractions of BASELINE configs 1, 3,
                4 and 5, plus the device quantiser and the reference-layout import on config 5;
  "ref_sweep"   (N=1) the reference's headline shape table (M=2048, FP16 out, its 36 measured
                (N, K) rows) timed its way, each row against the reference's published MI350X
                latency, with a count-weighted and a geometric-mean speed-up (--ref-sweep prints
                it alone, one line per shape; --no-ref-sweep skips it).

Timing: W untimed warm-up steps; then exactly K steps between a barrier + synchronize on each
side; before every timed step a 256 MiB buffer is written to flush the 126 MB L2, and each
step's GEMM is bracketed by CUDA events on the launching stream; ms_per_step is the mean over
the K steps, maximised over ranks. Clocks are sampled through NVML during the timed region.

Extra keys: "timing_as_reference" repeats the measurement with the reference's own convention
(8 warm-ups, 20 back-to-back calls, best of 4, no flush); --vs-cublas adds "vs_cublas_mxfp8",
cuBLASLt's block-scaled MXFP8 GEMM on the same shape (burst, interleaved, and sustained);
--import-only times just the device import of reference-layout weights (a small command for ncu).

--impl reference times the reference's own CPU GEMM (mxfp6_gemm_ref, compiled from its sources
into oracle/_ref) on the host cores, on a bounded row sample of the same workload and the same
operands; rank 0 only. That arm loads no part of this library: its operands come from the numpy
generator below (and, for config 5, the reference's own quantiser).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG_DIR = os.path.join(ROOT, "mxfp6-gemm_b200")

CONFIGS = {
    # name: (M, N, K, kind, exp_range, out)
    "cfg1": (256, 256, 512, "codes", (120, 134), "F32"),
    "cfg2": (8192, 8192, 8192, "codes", (118, 136), "F16"),
    "cfg3": (2048, 1024, 105728, "codes", (118, 136), "F16"),
    "cfg4": (2048, 6144, 16128, "codes", (118, 136), "BF16"),
    "cfg5": (4096, 28672, 8192, "normal", None, "BF16"),
}
CONFIG_DESC = {
    "cfg1": "MXFP6 GEMM M=256 N=256 K=512, FP32 output",
    "cfg2": "MXFP6 GEMM M=8192 N=8192 K=8192, FP16 output",
    "cfg3": "MXFP6 GEMM M=2048 N=1024 K=105728, FP16 output, split-K",
    "cfg4": "MXFP6 GEMM M=2048 N=6144 K=16128, BF16 output",
    "cfg5": "LLM FFN up-projection MXFP6 GEMM M=4096 N=28672 K=8192, BF16 output",
}
CFG5_SIGMA = (1.0, 0.02)  # A activation-like N(0, 1), B weight-like N(0, 0.02)
METRIC = "MXFP6 GEMM TFLOPS (2*M*N*K / device time)"
L2_FLUSH_BYTES = 256 << 20
L2_NOTE = "256 MiB buffer written before every timed step (L2 flushed)"
E2E_ROW_CHUNKS = 8  # default row chunks of A (and of D) in the end-to-end step
CUDA_MEMCPY_D2H = 2
# DRAM bytes (read + write) per launch of the dominant kernel, from one ncu capture of this
# bench's own command (profiles/gemm_mxfp6_sm100_pair_cfg2.md); None where not captured yet.
# DRAM bytes (read + write) of the dominant kernel per launch, from one ncu capture each (the
# summaries under profiles/ give the commands): cfg2, cfg3 (the banded split's pair kernel, without
# the reduce) and cfg4 with the current kernel, cfg5 with the same tiling and schedule.
NCU_TRAFFIC_BYTES = {"cfg2": 163_994_112 + 112_266_240, "cfg3": 290_432_768 + 10_324_736,
                     "cfg4": 202_283_776 + 30_461_952, "cfg5": 251_785_216 + 236_046_592}
NOMINAL_FP6_TFLOPS = 4500.0  # B200 dense FP8/FP6 tensor rate, nominal (no sparsity)
SEED_A, SEED_B = 1000, 2000  # operand seeds (B: plus the rank of its shard)


def kpad(K: int) -> int:
    return (K + 127) // 128 * 128


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["bf16_tflops"]), float(p["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 1590.0, 6650.0, "fallback"


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while running."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
        0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
        0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
    }

    def __init__(self, index: int):
        self.samples, self.reasons, self.max_mhz = [], 0, None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nvml = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:  # NVML missing: report no clocks rather than fail the bench
            self.nvml = None

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nvml.nvmlDeviceGetClockInfo(self.h, self.nvml.NVML_CLOCK_SM))
                self.reasons |= self.nvml.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            except Exception:
                pass
            time.sleep(0.005)

    def __enter__(self):
        if self.nvml:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._thread:
            self._thread.join()

    def summary(self):
        if not self.nvml:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml_unavailable"], "samples": 0}
        names = [n for b, n in self.REASONS.items() if self.reasons & b and n != "gpu_idle"]
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": names, "samples": len(self.samples)}


def e2e_upload_order(n_a, n_b, bytes_a, bytes_b):
    """Order of the end-to-end step's uploads: B chunk 0 first, then A while fewer A bytes than B
    bytes are up (B on a tie), so that the computable D blocks (one per pair of an A chunk and a
    B chunk already up) grow about as fast as possible per byte sent."""
    order, na, nb = [], 0, 0
    while na < n_a or nb < n_b:
        take_a = nb > 0 and na < n_a and (nb == n_b or nb * bytes_b > na * bytes_a)
        if take_a:
            order.append(("A", na))
            na += 1
        else:
            order.append(("B", nb))
            nb += 1
    return order


def cudart_memcpy2d_async():
    """cudaMemcpy2DAsync from the CUDA runtime the library is linked against (one pitched copy
    per D block; torch has no pitched host copy)."""
    import ctypes

    f = ctypes.CDLL("libcudart.so.12").cudaMemcpy2DAsync
    f.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t,
                  ctypes.c_size_t, ctypes.c_int, ctypes.c_void_p]
    f.restype = ctypes.c_int
    return f


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


# ---- synthetic operands (numpy; shared by both arms) ----------------------------------------------

def synth_codes(M, N, K, seed, exp_range):
    """Seeded E2M3 codes uniform over all 64 codes (the packed bytes are then uniform random
    bytes) and E8M0 exponents uniform in exp_range, in this library's host layouts: A packed
    [M][3Kp/4], B^T packed [N][3Kp/4], raw scales [rows][Kp/32]; a K tail past K is zero codes.
    Draw order A, B^T, sA, sB from one generator (the same draws as the package's
    synth.make_operands(kind="codes"), which the parity tests use)."""
    Kp = kpad(K)
    rb = Kp * 3 // 4
    rng = np.random.default_rng(seed)
    A = rng.integers(0, 256, (M, rb), dtype=np.uint8)
    Bt = rng.integers(0, 256, (N, rb), dtype=np.uint8)
    lo, hi = exp_range
    sA = rng.integers(lo, hi + 1, (M, Kp // 32), dtype=np.uint8)
    sB = rng.integers(lo, hi + 1, (N, Kp // 32), dtype=np.uint8)
    if K < Kp:
        A[:, K * 3 // 4:] = 0
        Bt[:, K * 3 // 4:] = 0
    return A, sA, Bt, sB


def synth_normal_rows(rows, K, seed, sigma, quantize):
    """rows x K floats ~ N(0, sigma), quantised per 32-block with max-abs E8M0 scaling by
    `quantize` (the reference's quantize_to_mxfp6, or this library's bit-identical one)."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((rows, K), dtype=np.float32) * np.float32(sigma)
    return quantize(x)


def bench_config(cfg_name, world, shards):
    """The `config` object of a line; both arms print the same one for the same arguments."""
    M, N, K, _, _, out = CONFIGS[cfg_name]
    n_per = N // shards if shards > 1 else N
    n_total = n_per * shards if shards > 1 else n_per * world
    workload = CONFIG_DESC[cfg_name]
    if world > 1:
        workload += f", N-sharded over {world} GPUs (per-GPU shard N={n_per})"
    if world == 1 and shards > 1:
        workload += f", the shard of one GPU out of {shards} (N={n_per} of {n_total})"
    return {"workload": workload, "M": M, "N_per_gpu": n_per, "N_total": n_total, "K": K, "out": out,
            "parallelism": f"N-sharded x{world}, no collective on the GEMM path", "l2": L2_NOTE}


# ---- reference arm: the reference's CPU GEMM on the host cores ------------------------------------

def _cpu_threads(N, K):
    """All host threads, capped so that each thread's private dequantised copy of B (the
    reference's mxfp6_gemm_ref dequantises both operands per call) fits in available memory."""
    threads = os.cpu_count() or 1
    try:
        avail = os.sysconf("SC_AVPHYS_PAGES") * os.sysconf("SC_PAGE_SIZE")
    except (ValueError, OSError):
        avail = 16 << 30
    per_thread = N * K * 4 + 64 * K * 4
    return max(1, min(threads, int(avail * 0.5 // per_thread)))


_CPU_OPS = {}


def _cpu_operands(cfg_name, n_cols):
    """The GPU arm's operands for rank 0: A (seed SEED_A) and the first B^T shard (seed SEED_B),
    with raw scales, from the numpy generator; config 5 is quantised by the reference's own
    quantize_to_mxfp6 (oracle/_ref) or, where that is not built, the C restatement."""
    key = (cfg_name, n_cols)
    if key not in _CPU_OPS:
        M, N, K, kind, er, _ = CONFIGS[cfg_name]
        if kind == "codes":
            A, sA, _, _ = synth_codes(M, 128, K, SEED_A, er)
            _, _, Bt, sB = synth_codes(128, n_cols, K, SEED_B, er)
        else:
            sys.path.insert(0, os.path.join(ROOT, "oracle"))
            from oracle import Oracle, Reference, reference_available
            q = Reference().quantize if reference_available() else Oracle().quantize
            A, sA = synth_normal_rows(M, K, SEED_A, CFG5_SIGMA[0], q)
            Bt, sB = synth_normal_rows(n_cols, K, SEED_B, CFG5_SIGMA[1], q)
        _CPU_OPS[key] = (A, sA, Bt, sB)
    return _CPU_OPS[key]


def cpu_reference_sample(cfg_name, n_cols=None, target_s=10.0, threads=None, rows_override=None):
    """Time mxfp6_gemm_ref (oracle/_ref, the reference's own CPU path; else the C restatement)
    on a row sample of the config: `rows` rows of A against all n_cols columns of B, sized to
    about target_s."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    from oracle import Oracle, Reference, reference_available

    M, N, K, _, _, _ = CONFIGS[cfg_name]
    n_cols = n_cols or N
    threads = threads or _cpu_threads(n_cols, K)
    A, sA, Bt, sB = _cpu_operands(cfg_name, n_cols)
    Kp = kpad(K)
    if reference_available() and Kp == K:
        ref, kind_s = Reference(), "reference"

        def run(rows):
            return ref.gemm(A[:rows], sA[:rows], Bt, sB, K, threads=threads)
    else:
        o, kind_s = Oracle(), "port"

        def run(rows):
            return o.gemm(A[:rows], sA[:rows], Bt, sB, Kp, threads=threads)

    if rows_override is None:
        # A warm-up call, then two timed sizes separate the per-call cost (each call dequantises
        # all of B per thread) from the per-row cost, so the sample lands near target_s.
        run(min(M, threads))
        r1, r2 = min(M, 4 * threads), min(M, 16 * threads)
        t0 = time.perf_counter()
        run(r1)
        t1 = time.perf_counter() - t0
        t0 = time.perf_counter()
        run(r2)
        t2 = time.perf_counter() - t0
        per_row = (t2 - t1) / (r2 - r1) if r2 > r1 and t2 > t1 else t2 / max(r2, 1)
        fixed = max(0.0, t2 - per_row * r2)
        rows = int((target_s - fixed) / max(per_row, 1e-9))
        rows = max(r2, min(M, rows // threads * threads if rows >= threads else rows))
    else:
        rows = min(rows_override, M)
    t0 = time.perf_counter()
    run(rows)
    dt = time.perf_counter() - t0
    tflops = 2.0 * rows * n_cols * K / dt / 1e12
    sample = (f"{rows} of {M} rows of A x all {n_cols} columns of B, K={K} "
              f"({2.0 * rows * n_cols * K / 1e9:.1f} GFLOP) in {dt:.2f} s on {threads} threads")
    return tflops, kind_s, threads, sample, rows


def run_reference_arm(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    shards = world if args.strong else args.shard_of
    config = bench_config(args.config, world, shards)
    n_cols, K = config["N_per_gpu"], config["K"]
    threads = _cpu_threads(n_cols, K)
    # one calibration pass picks the row sample, then K timed steps of that sample
    _, kind_s, cores, sample, rows = cpu_reference_sample(
        args.config, n_cols, target_s=min(args.ref_seconds, 150.0 / max(1, args.steps + args.warmup)),
        threads=threads)
    for _ in range(max(0, min(args.warmup, 1) - 1)):
        cpu_reference_sample(args.config, n_cols, threads=threads, rows_override=rows)
    vals = []
    for _ in range(args.steps):
        v, kind_s, cores, sample, _ = cpu_reference_sample(args.config, n_cols, threads=threads,
                                                           rows_override=rows)
        vals.append(v)
    value = statistics.mean(vals)
    flops_step = 2.0 * rows * n_cols * K
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOPS", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": flops_step / (value * 1e12) * 1e3,
        "higher_is_better": True, "scaling": "strong" if args.strong else "weak", "vs_baseline": None,
        "dtype": "fp6_e2m3 x fp6_e2m3 -> f32 accumulate",
        "data": "synthetic (seeded E2M3 codes uniform over 64 codes, E8M0 exponents per BASELINE)",
        "config": config,
        "cpu_baseline": {"value": value, "unit": "TFLOPS", "cores": cores, "kind": kind_s,
                         "sample": f"each step: {sample}"},
        "e2e": {"value": value, "unit": "TFLOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---- our arm ----------------------------------------------------------------------------------------

def run_vs_cublas(M, N, K, step, stream, flush, dev, rounds=6, burst=8, sustain_s=1.0):
    """Context for the roofline: cuBLASLt's block-scaled MXFP8 GEMM (E4M3 operands, one E8M0
    scale per 32 elements, the same tcgen05 instruction family and tensor rate as FP6) on the same
    M, N, K with BF16 output, through torch's scaled_mm. Burst: the two kernels alternate in
    rounds of `burst` L2-flushed launches so that clock and power drift affects both alike.
    Sustained: each runs back to back for `sustain_s` seconds under NVML clock sampling (B200
    settles under its power cap)."""
    import torch
    import torch.nn.functional as F

    try:
        a8 = (torch.randn(M, K, device=dev) * 0.5).to(torch.float8_e4m3fn)
        b8 = (torch.randn(N, K, device=dev) * 0.5).to(torch.float8_e4m3fn).t()
        nsa = (M + 127) // 128 * 128 * ((K // 32 + 3) // 4 * 4)
        nsb = (N + 127) // 128 * 128 * ((K // 32 + 3) // 4 * 4)
        sa = torch.full((nsa,), 127, dtype=torch.uint8, device=dev).view(torch.float8_e8m0fnu)
        sb = torch.full((nsb,), 127, dtype=torch.uint8, device=dev).view(torch.float8_e8m0fnu)

        def mx8():
            return F.scaled_mm(a8, b8, sa, F.ScalingType.BlockWise1x32, sb, F.ScalingType.BlockWise1x32,
                               F.SwizzleType.SWIZZLE_32_4_4, F.SwizzleType.SWIZZLE_32_4_4,
                               output_dtype=torch.bfloat16)

        for _ in range(3):
            mx8()
        torch.cuda.synchronize()
    except Exception as e:  # no MX support in this torch / cuBLASLt: report, do not fail the bench
        return {"unavailable": f"cuBLASLt MXFP8 via torch scaled_mm: {e!r}"[:300]}

    fns = {"ours": step, "cublas_mxfp8": mx8}
    times = {k: [] for k in fns}
    for r in range(rounds):
        for name in (fns if r % 2 == 0 else reversed(list(fns))):
            for i in range(burst):
                flush.fill_(i & 0xFF)
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                fns[name]()
                e1.record(stream)
                torch.cuda.synchronize()
                times[name].append(e0.elapsed_time(e1))
    flop = 2.0 * M * N * K
    out = {"what": "cuBLASLt block-scaled MXFP8 (E4M3 x E4M3, E8M0 per 32, BF16 out) on the same M, N, K",
           "burst": {}, "sustained": {}}
    for name, ts in times.items():
        med = statistics.median(ts)
        out["burst"][name] = {"median_ms": med, "tflops": flop / (med * 1e-3) / 1e12}
    out["burst"]["ours_over_cublas"] = out["burst"]["ours"]["tflops"] / out["burst"]["cublas_mxfp8"]["tflops"]
    for name, fn in fns.items():
        torch.cuda.synchronize()
        n, t0 = 0, time.time()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        with ClockSampler(dev.index or 0) as clk:
            e0.record(stream)
            while time.time() - t0 < sustain_s:
                for _ in range(25):
                    fn()
                n += 25
                e1.record(stream)
                e1.synchronize()
            e1.record(stream)
            torch.cuda.synchronize()
        per = e0.elapsed_time(e1) / n
        out["sustained"][name] = {"ms": per, "tflops": flop / (per * 1e-3) / 1e12, "clocks": clk.summary()}
    out["sustained"]["ours_over_cublas"] = (out["sustained"]["ours"]["tflops"]
                                            / out["sustained"]["cublas_mxfp8"]["tflops"])
    return out


def time_import_leg(lib, N, K, rb, stream, dev, reps=20):
    """Device import of B^T [N x K] laid out as the reference lays out weights (gfx950
    preshuffle_B, K padded to a multiple of 192) into this library's rows of rb bytes. The import
    is a byte permutation, so random bytes time it as well as real weights."""
    import torch

    kp_ref = (K + 191) // 192 * 192
    ref_b = torch.randint(0, 256, ((N // 32) * (kp_ref // 64) * 1536,), dtype=torch.uint8, device=dev)
    imp_b = torch.empty((N, rb), dtype=torch.uint8, device=dev)
    for _ in range(3):
        assert lib.import_ref_B_device(ref_b, N, kp_ref, imp_b, rb, stream=stream) == lib.OK
    i0 = torch.cuda.Event(enable_timing=True)
    i1 = torch.cuda.Event(enable_timing=True)
    i0.record(stream)
    for _ in range(reps):
        lib.import_ref_B_device(ref_b, N, kp_ref, imp_b, rb, stream=stream)
    i1.record(stream)
    torch.cuda.synchronize()
    ms = i0.elapsed_time(i1) / reps
    nbytes = ref_b.numel() + imp_b.numel()
    _, hbm_peak, basis = load_peaks()
    return {"what": f"B^T [{N}x{K}] from the reference's preshuffle_B layout (Kp_ref={kp_ref}) to this "
                    f"library's rows of {rb} bytes, on the device",
            "ms": ms, "gbs": nbytes / (ms * 1e-3) / 1e9, "frac_hbm": nbytes / (ms * 1e-3) / 1e9 / hbm_peak,
            "peak_basis": f"{basis} copy bandwidth {hbm_peak:.0f} GB/s", "bytes_per_launch": nbytes}


def _torch_out(lib, torch, ot):
    return {lib.OutType.F32: torch.float32, lib.OutType.F16: torch.float16, lib.OutType.BF16: torch.bfloat16}[ot]


def codes_device_operands(lib, torch, cfg_name, n_cols, b_seed, dev):
    """A (seed SEED_A) and an n_cols-row B^T (seed b_seed) of a "codes" config on the device, scales
    in the GEMM's atom layout."""
    M, _, K, _, er, _ = CONFIGS[cfg_name]
    A, sA, _, _ = synth_codes(M, 128, K, SEED_A, er)
    _, _, Bt, sB = synth_codes(128, n_cols, K, b_seed, er)
    Kp = kpad(K)
    return (torch.from_numpy(A).to(dev), torch.from_numpy(lib.preprocess_scale(sA, M, Kp)).to(dev),
            torch.from_numpy(Bt).to(dev), torch.from_numpy(lib.preprocess_scale(sB, n_cols, Kp)).to(dev))


def cfg5_device_operands(lib, torch, dev, stream):
    """BASELINE config 5 on the device: A ~ N(0, 1) [M][K] and B^T ~ N(0, 0.02) [N][K] from torch's
    seeded generator, quantised per 32-block with max-abs E8M0 scaling by this library's device
    quantiser (bit-identical to quantize_to_mxfp6), scales in the GEMM's atom layout."""
    M, N, K, _, _, _ = CONFIGS["cfg5"]
    Kp = kpad(K)
    out = []
    for rows, seed, sigma in ((M, SEED_A, CFG5_SIGMA[0]), (N, SEED_B, CFG5_SIGMA[1])):
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        x = torch.randn((rows, K), generator=g, device=dev, dtype=torch.float32) * sigma
        q = torch.empty((rows, Kp * 3 // 4), dtype=torch.uint8, device=dev)
        s = torch.empty(lib.tiled_scale_bytes(rows, Kp), dtype=torch.uint8, device=dev)
        rc = lib.quantize_device(x, rows, K, q, s, True, stream=stream)
        if rc != lib.OK:
            raise RuntimeError(f"device quantiser failed: {rc}")
        del x
        out += [q, s]
    torch.cuda.synchronize()
    return out  # A, sA, Bt, sB


def workspace(lib, torch, M, N, Kp, ot, dev):
    """Workspace for this output type's route (the type-free query is the max over types)."""
    wsb = lib.gemm_workspace_size(M, N, Kp, ot)
    return (torch.empty(wsb, dtype=torch.uint8, device=dev) if wsb else None), wsb


def timed_calls(torch, fn, steps, warmup, flush, stream):
    """Per-call device times (ms): `warmup` untimed calls, then `steps` calls, each after an L2
    flush, between CUDA events on the launching stream."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for i, (a, b) in enumerate(ev):
        flush.fill_(i & 0xFF)
        a.record(stream)
        fn()
        b.record(stream)
    torch.cuda.synchronize()
    return [a.elapsed_time(b) for a, b in ev]


def roofline_fields(M, N, K, Kp, out_bytes, ms, wsb):
    bf16_peak, _, basis = load_peaks()
    peak = 2.0 * bf16_peak
    tflops = 2.0 * M * N * K / (ms * 1e-3) / 1e12
    algo_bytes = (M + N) * Kp * 3 // 4 + (M + N) * (Kp // 32) + M * N * out_bytes
    return {"tflops": tflops, "frac": tflops / peak, "frac_of_nominal_fp6_dense": tflops / NOMINAL_FP6_TFLOPS,
            "peak": peak, "peak_basis": f"2 x {basis} cuBLAS bf16 dense ({bf16_peak:.1f} TFLOP/s)",
            "algorithmic_bytes": algo_bytes, "algorithmic_gbs": algo_bytes / (ms * 1e-3) / 1e9,
            "splitk_workspace_bytes": 2 * wsb}


def per_config_leg(lib, torch, dev, stream, flush, steps, warmup, skip):
    """N=1: BASELINE configs 1, 3 and 4 timed like the headline (config 5 comes from the strong
    leg, which at N=1 is config 5 on one GPU)."""
    out = {}
    for name in ("cfg1", "cfg3", "cfg4"):
        if name == skip:
            continue
        M, N, K, _, _, out_name = CONFIGS[name]
        Kp = kpad(K)
        rb = Kp * 3 // 4
        ot = lib.OutType[out_name]
        A, sA, Bt, sB = codes_device_operands(lib, torch, name, N, SEED_B, dev)
        D = torch.empty((M, N), dtype=_torch_out(lib, torch, ot), device=dev)
        ws, wsb = workspace(lib, torch, M, N, Kp, ot, dev)

        def call_on(st):
            lib.gemm(ot, M, N, Kp, A, Bt, sA, sB, D, rb, rb, ws, wsb, stream=st)

        def call():
            call_on(stream)

        per = timed_calls(torch, call, steps, warmup, flush, stream)
        err, status = lib.last_error(), lib.device_status()
        ms = sum(per) / len(per)
        entry = {"workload": CONFIG_DESC[name], "M": M, "N": N, "K": K, "out": out_name,
                 "route": lib.route(ot, M, N, Kp), "ms": ms, "best_ms": min(per), "steps": steps,
                 "error": err, "device_status": status}
        entry.update(roofline_fields(M, N, K, Kp, D.element_size(), ms, wsb))
        if name in NCU_TRAFFIC_BYTES:
            entry["traffic"] = NCU_TRAFFIC_BYTES[name]  # dominant kernel's DRAM bytes per launch (ncu)
        if name == "cfg1":
            entry["back_to_back"] = back_to_back_per_call(torch, call_on, stream)
            entry["back_to_back"].update(cpp_cfg1_per_call())
        out[name] = entry
        del A, sA, Bt, sB, D, ws
    return out


def build_cpp_caller(tmp):
    """Compile the C++ drop-in caller of the tests (g++ against the public headers, linked to this
    library) into `tmp`; returns the executable's path."""
    import subprocess
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    lib_dir = os.path.join(PKG_DIR, "lib")
    exe = os.path.join(tmp, "drop_in_caller")
    cmd = ["g++", "-std=c++17", "-O2", "-I", os.path.join(ROOT, "include"), "-I", os.path.join(cuda, "include"),
           os.path.join(ROOT, "tests", "cpp", "drop_in_caller.cpp"), "-o", exe, "-L", lib_dir, "-lmxfp6gemm",
           f"-Wl,-rpath,{lib_dir}", "-L", os.path.join(cuda, "lib64"), "-lcudart",
           f"-Wl,-rpath,{os.path.join(cuda, 'lib64')}"]
    subprocess.run(cmd, check=True, capture_output=True, timeout=120)
    return exe


def cpp_time(exe, shape=None):
    """Per-call µs of the C++ caller's `time` mode (cfg1, or `shape` = (M, N, K, OUT))."""
    import re
    import subprocess
    argv = [exe, "time"] + ([str(x) for x in shape] if shape else [])
    out = subprocess.run(argv, check=True, capture_output=True, text=True, timeout=120).stdout
    m = re.search(r"back-to-back from C\+\+: ([0-9.]+) us per call", out)
    if not m:
        raise RuntimeError(out[-200:])
    return float(m.group(1))


def cpp_cfg1_per_call():
    """Config 1 timed from C++ through the reference's own API (mxfp6::gemm on the legacy default
    stream, 20 back-to-back calls, best of 4: the reference harness's convention): the C++
    drop-in caller of the tests, compiled with g++ against the public headers, in its `time` mode."""
    import subprocess
    import tempfile
    with tempfile.TemporaryDirectory() as tmp:
        try:
            return {"cpp_eager_us": cpp_time(build_cpp_caller(tmp))}
        except (OSError, RuntimeError, subprocess.SubprocessError) as e:
            return {"cpp_unavailable": repr(e)[:200]}


def back_to_back_per_call(torch, call_on, stream, calls=20, reps=4):
    """Per-call time of `calls` back-to-back calls between two events, best of `reps` (the
    reference's own convention for its launch-bound floor, tests/test_gemm.cpp:32-52): issued from
    Python (host enqueue included where it exceeds the device time), and replayed from a CUDA graph
    of the same calls (device time only; consecutive kernels overlap their set-up through
    programmatic dependent launch)."""
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    eager = []
    for _ in range(reps):
        e0.record(stream)
        for _ in range(calls):
            call_on(stream)
        e1.record(stream)
        e1.synchronize()
        eager.append(e0.elapsed_time(e1) * 1e3 / calls)
    out = {"calls": calls, "eager_us": min(eager)}
    try:
        cs = torch.cuda.Stream()  # capture needs a stream other than the legacy default one
        cs.wait_stream(stream)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=cs):
            for _ in range(calls):
                call_on(cs)
        graph = []
        with torch.cuda.stream(cs):  # replay() launches on the current stream
            for _ in range(reps + 1):
                e0.record(cs)
                g.replay()
                e1.record(cs)
                e1.synchronize()
                graph.append(e0.elapsed_time(e1) * 1e3 / calls)
        out["graph_us"] = min(graph[1:])
        del g
    except Exception as e:  # capture unavailable: report the eager figure alone
        out["graph_unavailable"] = repr(e)[:200]
    return out


def device_legs_cfg5(lib, torch, dev, stream, A, Bt):
    """The steps either side of the config-5 GEMM on the device: quantising the activations, and
    importing weights held in the reference's (gfx950) preprocessed layout."""
    M, N, K, _, _, _ = CONFIGS["cfg5"]
    Kp = kpad(K)
    rb = Kp * 3 // 4
    _, hbm_peak, basis = load_peaks()
    xf = torch.randn((M, K), device=dev, dtype=torch.float32)
    qa = torch.empty((M, rb), dtype=torch.uint8, device=dev)
    qs = torch.empty(lib.tiled_scale_bytes(M, Kp), dtype=torch.uint8, device=dev)
    for _ in range(3):
        assert lib.quantize_device(xf, M, K, qa, qs, True, stream=stream) == lib.OK
    q0 = torch.cuda.Event(enable_timing=True)
    q1 = torch.cuda.Event(enable_timing=True)
    reps = 20
    q0.record(stream)
    for _ in range(reps):
        lib.quantize_device(xf, M, K, qa, qs, True, stream=stream)
    q1.record(stream)
    torch.cuda.synchronize()
    qms = q0.elapsed_time(q1) / reps
    qbytes = M * K * 4 + M * K * 3 // 4 + M * K // 32
    quant = {"what": f"quantize A [{M}x{K}] fp32 -> MXFP6 + tiled scales on the device", "ms": qms,
             "gbs": qbytes / (qms * 1e-3) / 1e9, "frac_hbm": qbytes / (qms * 1e-3) / 1e9 / hbm_peak,
             "peak_basis": f"{basis} copy bandwidth {hbm_peak:.0f} GB/s"}
    del xf, qa, qs
    return quant, time_import_leg(lib, N, K, rb, stream, dev)


def gather_legs(lib, torch, dist, dev, stream, flush, rank, world, ot, tdt, M, Ng, Kp, rb, A, Bt_r, sA, sB_r,
                D_r, ws, wsb, shard_ms, D_ref):
    """The optional gather of the column shards into every rank's row-major D[M][world*Ng]:
    NCCL all-gather of the finished shards, and the fused alternative (mxfp6_gemm_gather: the
    GEMM's epilogue stores each D chunk into every rank's gathered D through CUDA IPC peer
    pointers). Both are checked bit for bit against D_ref, the unsplit GEMM of this rank."""
    from mxfp6_b200.shard import assemble_columns

    bits = torch.int32 if tdt == torch.float32 else torch.int16
    gathered = torch.empty((world, M, Ng), dtype=tdt, device=dev)
    for _ in range(2):
        dist.all_gather_into_tensor(gathered, D_r)
    torch.cuda.synchronize()
    dist.barrier()
    g0 = torch.cuda.Event(enable_timing=True)
    g1 = torch.cuda.Event(enable_timing=True)
    reps = 5
    g0.record(stream)
    for _ in range(reps):
        dist.all_gather_into_tensor(gathered, D_r)
    g1.record(stream)
    torch.cuda.synchronize()
    t = torch.tensor([g0.elapsed_time(g1) / reps], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ag_ms = float(t.item())
    nbytes = D_r.numel() * D_r.element_size()
    same = torch.equal(assemble_columns(gathered).view(bits), D_ref.view(bits))
    f = torch.tensor([1 if same else 0], device=dev, dtype=torch.int32)
    dist.all_reduce(f, op=dist.ReduceOp.MIN)
    out = {"nccl_allgather": {"ms": ag_ms, "bytes_per_rank": nbytes,
                              "bus_gbs": nbytes * (world - 1) / (ag_ms * 1e-3) / 1e9,
                              "gemm_then_allgather_ms": shard_ms + ag_ms,
                              "assembled_equals_one_gpu_D": bool(f.item() == 1),
                              "what": "NCCL all_gather_into_tensor of the [M][N/g] shards, reassembled row-major"}}
    del gathered

    fused = {"unavailable": "fused gather skipped"}
    ok_local, handle = 1, (None, 0)
    gathered2 = torch.empty((M, Ng * world), dtype=tdt, device=dev)
    try:
        handle = lib.ipc_export(gathered2)
    except Exception as e:  # reported, and every rank skips together
        ok_local, fused = 0, {"unavailable": f"ipc export: {e}"}
    handles = [None] * world
    dist.all_gather_object(handles, handle)
    dsts, bases = [], []
    for r in range(world):
        if r == rank:
            dsts.append(gathered2.data_ptr())
        elif ok_local and handles[r][0] is not None:
            try:
                base, ptr = lib.ipc_import(*handles[r])
                bases.append(base)
                dsts.append(ptr)
            except Exception as e:
                ok_local, fused = 0, {"unavailable": f"ipc import: {e}"}
        else:
            ok_local = 0
    flag = torch.tensor([ok_local], device=dev, dtype=torch.int32)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    if int(flag.item()) == 1:
        def fstep():
            lib.gemm_gather(ot, M, Ng, Kp, A, Bt_r, sA, sB_r, dsts, Ng * world, rank * Ng, rb, rb, ws, wsb,
                            stream=stream)

        for _ in range(2):
            fstep()
        torch.cuda.synchronize()
        fail = torch.tensor([0 if lib.last_error() == lib.OK else 1], device=dev, dtype=torch.int32)
        dist.all_reduce(fail, op=dist.ReduceOp.MAX)
        if int(fail.item()) == 0:
            fts = []
            for i in range(reps):
                dist.barrier()
                flush.fill_(i & 0xFF)
                torch.cuda.synchronize()
                f0 = torch.cuda.Event(enable_timing=True)
                f1 = torch.cuda.Event(enable_timing=True)
                f0.record(stream)
                fstep()
                f1.record(stream)
                torch.cuda.synchronize()
                fts.append(f0.elapsed_time(f1))
            t = torch.tensor([sum(fts) / len(fts)], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            f_ms = float(t.item())
            dist.barrier()  # every rank's peer stores have landed
            same = torch.equal(gathered2.view(bits), D_ref.view(bits))
            sflag = torch.tensor([1 if same else 0], device=dev, dtype=torch.int32)
            dist.all_reduce(sflag, op=dist.ReduceOp.MIN)
            fused = {"ms": f_ms, "speedup_vs_gemm_then_allgather": (shard_ms + ag_ms) / f_ms,
                     "nvlink_bytes_per_rank": nbytes * (world - 1),
                     "equals_one_gpu_D": bool(sflag.item() == 1), "device_status": lib.device_status(),
                     "what": "mxfp6_gemm_gather: the shard GEMM's epilogue stores each D chunk into all ranks' "
                             "gathered [M][N] outputs through CUDA IPC peer pointers"}
        else:
            fused = {"unavailable": "mxfp6_gemm_gather rejected the call on some rank"}
    torch.cuda.synchronize()
    dist.barrier()
    for base in bases:
        lib.ipc_close(base)
    dist.barrier()
    out["fused_gather"] = fused
    del gathered2
    return out


def strong_leg(lib, torch, dist, dev, stream, flush, rank, world, steps, warmup, with_gather, with_device_legs):
    """BASELINE config 5 with B and D split column-parallel over the ranks (strong scaling): rank r
    computes D[:, r*N/g : (r+1)*N/g] from all of A and its rows of B^T; no collective on the GEMM
    path. Timed like the headline (flushed L2, events, max over ranks). Each rank also runs the
    unsplit GEMM on its GPU, for the efficiency and as the reference its shard must equal bit for
    bit."""
    M, N, K, _, _, out_name = CONFIGS["cfg5"]
    Kp = kpad(K)
    rb = Kp * 3 // 4
    ot = lib.OutType[out_name]
    tdt = _torch_out(lib, torch, ot)
    A, sA, Bt, sB = cfg5_device_operands(lib, torch, dev, stream)
    Ng = N // world
    atoms = Kp // 128 * 512  # scale bytes per 128 rows
    Bt_r = Bt[rank * Ng:(rank + 1) * Ng]
    sB_r = sB[rank * Ng // 128 * atoms:(rank + 1) * Ng // 128 * atoms]
    D_r = torch.empty((M, Ng), dtype=tdt, device=dev)
    ws_r, wsb_r = workspace(lib, torch, M, Ng, Kp, ot, dev)

    def shard():
        lib.gemm(ot, M, Ng, Kp, A, Bt_r, sA, sB_r, D_r, rb, rb, ws_r, wsb_r, stream=stream)

    for _ in range(warmup):
        shard()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(dev.index or 0) as clk:
        per = timed_calls(torch, shard, steps, 0, flush, stream)
    if world > 1:
        dist.barrier()
    ms_local = sum(per) / len(per)
    err, status = lib.last_error(), lib.device_status()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    ms = max_over_ranks(ms_local)
    total = 2.0 * M * N * K / (ms * 1e-3) / 1e12
    entry = {"workload": CONFIG_DESC["cfg5"] + f", B and D split column-parallel over {world} GPU(s)",
             "M": M, "N_total": N, "N_per_gpu": Ng, "K": K, "out": out_name, "route": lib.route(ot, M, Ng, Kp),
             "ms": ms, "total_tflops": total, "per_gpu_tflops": total / world, "steps": steps,
             "clocks": clk.summary(), "error": err, "device_status": status}
    entry.update({k: v for k, v in roofline_fields(M, Ng, K, Kp, D_r.element_size(), ms, wsb_r).items()
                  if k not in ("tflops",)})
    if world == 1:
        D_full = D_r
        entry["traffic"] = NCU_TRAFFIC_BYTES["cfg5"]  # the pair kernel's DRAM bytes per launch (ncu)
        entry["one_gpu"] = {"ms": ms, "tflops": total}
        entry["efficiency_vs_one_gpu"] = 1.0
    else:
        D_full = torch.empty((M, N), dtype=tdt, device=dev)
        ws_f, wsb_f = workspace(lib, torch, M, N, Kp, ot, dev)

        def full():
            lib.gemm(ot, M, N, Kp, A, Bt, sA, sB, D_full, rb, rb, ws_f, wsb_f, stream=stream)

        per_f = timed_calls(torch, full, steps, warmup, flush, stream)
        ms_f = max_over_ranks(sum(per_f) / len(per_f))
        tf1 = 2.0 * M * N * K / (ms_f * 1e-3) / 1e12
        entry["one_gpu"] = {"ms": ms_f, "tflops": tf1, "route": lib.route(ot, M, N, Kp),
                            "how": "the unsplit GEMM on each rank's GPU, max over ranks"}
        entry["efficiency_vs_one_gpu"] = (total / world) / tf1
        bits = torch.int32 if tdt == torch.float32 else torch.int16
        same = torch.equal(D_r.view(bits), D_full[:, rank * Ng:(rank + 1) * Ng].contiguous().view(bits))
        f = torch.tensor([1 if same else 0], device=dev, dtype=torch.int32)
        dist.all_reduce(f, op=dist.ReduceOp.MIN)
        entry["shards_equal_one_gpu_D"] = bool(f.item() == 1)
        if with_gather:
            entry.update(gather_legs(lib, torch, dist, dev, stream, flush, rank, world, ot, tdt, M, Ng, Kp, rb,
                                     A, Bt_r, sA, sB_r, D_r, ws_r, wsb_r, ms, D_full))
        del ws_f
    if with_device_legs and world == 1:
        entry["quantize_device"], entry["import_ref_B_device"] = device_legs_cfg5(lib, torch, dev, stream, A, Bt)
    del A, sA, Bt, sB, D_r, D_full
    return entry


def run_ours(args):
    sys.path.insert(0, PKG_DIR)
    import torch
    import torch.distributed as dist

    import mxfp6_b200 as lib

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    M, N, K, kind, er, out_name = CONFIGS[args.config]
    # --strong: the config's N is the job's total, split over the ranks (strong scaling);
    # --shard-of G: run on this GPU the shard one rank of a G-GPU strong-scaled job holds.
    shards = world if args.strong else args.shard_of
    config = bench_config(args.config, world, shards)
    N = config["N_per_gpu"]
    ot = lib.OutType[out_name]
    Kp = kpad(K)
    rb = Kp * 3 // 4
    stream = torch.cuda.current_stream(dev)
    # A is replicated (same seed everywhere); B^T's shard differs per rank (column-parallel).
    if kind == "codes":
        A, sA, Bt, sB = codes_device_operands(lib, torch, args.config, N, SEED_B + rank, dev)
    else:
        A, sA, Bt_all, sB_all = cfg5_device_operands(lib, torch, dev, stream)
        r0 = rank if args.strong else 0
        atoms = Kp // 128 * 512
        Bt = Bt_all[r0 * N:(r0 + 1) * N].clone()
        sB = sB_all[r0 * N // 128 * atoms:(r0 + 1) * N // 128 * atoms].clone()
        del Bt_all, sB_all
    tdt = _torch_out(lib, torch, ot)
    D = torch.empty((M, N), dtype=tdt, device=dev)
    ws, wsb = workspace(lib, torch, M, N, Kp, ot, dev)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)

    def step():
        lib.gemm(ot, M, N, Kp, A, Bt, sA, sB, D, rb, rb, ws, wsb, stream=stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    assert lib.last_error() == lib.OK, lib.last_error_string()
    assert lib.device_status() == 0

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    launches0 = lib.launch_count()
    with ClockSampler(local) as clk:
        for i in range(args.steps):
            flush.fill_(i & 0xFF)
            starts[i].record(stream)
            step()
            ends[i].record(stream)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    launches = lib.launch_count() - launches0
    status = lib.device_status()
    per = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    ms = sum(per) / len(per)
    if world > 1:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    flops_rank = 2.0 * M * N * K
    value = flops_rank * world / (ms * 1e-3) / 1e12

    # ---- end to end through the C ABI with host buffers ----
    def e2e_leg():
        pinned = {k: v.cpu().pin_memory() for k, v in (("A", A), ("Bt", Bt), ("sA", sA), ("sB", sB))}
        # Two sets of device operands and results (and two pinned result buffers), used by
        # alternate steps, so that one step's uploads can run while the previous step's results
        # go down. Every step still moves all of its inputs up and all of its result down.
        sets = []
        for _ in range(2):
            sets.append({"A": torch.empty_like(A), "Bt": torch.empty_like(Bt), "sA": torch.empty_like(sA),
                         "sB": torch.empty_like(sB), "D": torch.empty_like(D),
                         "Dh": torch.empty((M, N), dtype=tdt).pin_memory(), "computed": None, "down": None})
        h2d = sum(p.numel() * p.element_size() for p in pinned.values())
        d2h = sets[0]["Dh"].numel() * sets[0]["Dh"].element_size()

        # A step's transfers and math overlap in a two-dimensional block pipeline. A is cut into
        # row chunks and B^T into row chunks (column chunks of B and D). The chunks go up on a copy
        # stream in an order that keeps D blocks coming as early as possible (e2e_upload_order); a
        # first block of D is computable after two chunks. Each block D[i, j] is one call of the
        # library's public entry on the compute stream as soon as A_i and B_j have landed:
        # mxfp6_gemm_gather with one destination (D's row i*mc) writes the block straight into D
        # (row stride N, first column j*nc). Each block goes back on a third stream, as a pitched
        # copy, as soon as it is computed. Consecutive steps use alternate buffer sets: a step's
        # uploads wait only until the GEMMs of the step before last (same set) have read their
        # operands, and its GEMMs until that step's result has gone down.
        s_up = torch.cuda.Stream(dev)
        s_down = torch.cuda.Stream(dev)
        ra = args.e2e_rows if args.e2e_rows > 0 and M % (128 * args.e2e_rows) == 0 else 1
        rc = args.e2e_cols if args.e2e_cols > 0 and N % (128 * args.e2e_cols) == 0 else 1
        mc, nc = M // ra, N // rc
        sa_chunk = (mc // 128) * (Kp // 128) * 512  # scale atoms are row-block major
        sb_chunk = (nc // 128) * (Kp // 128) * 512
        ws_c, wsb_c = workspace(lib, torch, mc, nc, Kp, ot, dev)  # a block's own route may split K
        order = e2e_upload_order(ra, rc, mc * rb, nc * rb)
        memcpy2d = cudart_memcpy2d_async()
        esz = sets[0]["Dh"].element_size()

        def e2e_step(st):
            if st["computed"] is not None:
                s_up.wait_event(st["computed"])  # the step before last has read this set's operands
            have_a, have_b, blocks = [], [], []
            with torch.cuda.stream(s_up):
                for kind_c, k in order:
                    if kind_c == "A":
                        st["A"][k * mc:(k + 1) * mc].copy_(pinned["A"][k * mc:(k + 1) * mc], non_blocking=True)
                        st["sA"][k * sa_chunk:(k + 1) * sa_chunk].copy_(
                            pinned["sA"][k * sa_chunk:(k + 1) * sa_chunk], non_blocking=True)
                    else:
                        st["Bt"][k * nc:(k + 1) * nc].copy_(pinned["Bt"][k * nc:(k + 1) * nc], non_blocking=True)
                        st["sB"][k * sb_chunk:(k + 1) * sb_chunk].copy_(
                            pinned["sB"][k * sb_chunk:(k + 1) * sb_chunk], non_blocking=True)
                    ev = torch.cuda.Event()
                    ev.record(s_up)
                    if kind_c == "A":
                        blocks += [(k, j, ev) for j in have_b]
                        have_a.append(k)
                    else:
                        blocks += [(i, k, ev) for i in have_a]
                        have_b.append(k)
            if st["down"] is not None:
                stream.wait_event(st["down"])  # the step before last's result has left this set's D
            done = []
            Dd = st["D"]
            for i, j, ev in blocks:
                stream.wait_event(ev)
                lib.gemm_gather(ot, mc, nc, Kp, st["A"][i * mc:], st["Bt"][j * nc:], st["sA"][i * sa_chunk:],
                                st["sB"][j * sb_chunk:], [Dd[i * mc:].data_ptr()], N, j * nc, rb, rb, ws_c, wsb_c,
                                stream=stream)
                ev = torch.cuda.Event()
                ev.record(stream)
                done.append((i, j, ev))
            st["computed"] = done[-1][2]
            Dh = st["Dh"]
            for i, j, ev in done:
                s_down.wait_event(ev)
                off = (i * mc * N + j * nc) * esz
                err = memcpy2d(Dh.data_ptr() + off, N * esz, Dd.data_ptr() + off, N * esz, nc * esz, mc,
                               CUDA_MEMCPY_D2H, s_down.cuda_stream)
                if err != 0:
                    raise RuntimeError(f"cudaMemcpy2DAsync failed: {err}")
            st["down"] = torch.cuda.Event()
            st["down"].record(s_down)

        def timed(n, pipelined):
            """ms per step over n steps, from an event on the compute stream before the first
            upload to one after the last result has landed in host memory."""
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            s_up.wait_event(e0)
            for k in range(n):
                e2e_step(sets[k % 2] if pipelined else sets[0])
                if not pipelined:  # the next step starts once this one's result is in host memory
                    s_up.wait_event(sets[0]["down"])
            for st in sets:
                if st["down"] is not None:
                    stream.wait_event(st["down"])
            e1.record(stream)
            torch.cuda.synchronize()
            return e0.elapsed_time(e1) / n

        e2e_steps = max(4, min(args.steps, 20))
        D_dev = D.clone()  # the device-timed result, to compare the end-to-end output with
        timed(2, True)
        bits = torch.int32 if tdt == torch.float32 else torch.int16
        e2e_same = min(float((st["Dh"].to(dev).view(bits) == D_dev.view(bits)).float().mean().item())
                       for st in sets)
        del D_dev
        if world > 1:
            dist.barrier()
        serial_ms = timed(e2e_steps, False)
        if world > 1:
            dist.barrier()
        e2e_ms = timed(e2e_steps, True)
        if world > 1:
            t = torch.tensor([e2e_ms, serial_ms], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e2e_ms, serial_ms = float(t[0].item()), float(t[1].item())
        e2e_value = flops_rank * world / (e2e_ms * 1e-3) / 1e12
        return {"value": e2e_value, "unit": "TFLOPS", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": e2e_ms, "bitwise_equal_to_device_run": e2e_same,
                "one_step_at_a_time": {"ms_per_step": serial_ms,
                                       "value": flops_rank * world / (serial_ms * 1e-3) / 1e12,
                                       "how": "each step's uploads start after the previous step's result "
                                              "is in host memory"},
                "path": f"pinned host -> H2D in {ra} row chunks of A and {rc} of B^T (interleaved, with their "
                        f"scales), overlapped with one C-ABI call (mxfp6_gemm_gather, one destination) per "
                        f"{mc}x{nc} block of D as soon as its chunks land, overlapped with a pitched D2H "
                        f"copy per block; consecutive steps on alternate buffer sets, so one step's uploads "
                        f"overlap the previous step's downloads"}

    e2e = None if args.no_e2e else e2e_leg()

    # ---- compact A (the reference's row stride 3K/4 with K % 128 != 0; loader-warp producer) ----
    compact = None
    if args.with_compact and world == 1 and K % 128 == 0 and K > 128:
        Kc = K - 32  # same Kp, so the same MMA work; A rows of 3*Kc/4 bytes
        rbc = Kc * 3 // 4
        Ac = A[:, :rbc].contiguous()
        Btc = Bt.clone()
        Btc[:, rbc:] = 0  # the recipe's zero B tail

        def cstep(w, wb):
            lib.gemm(ot, M, N, Kp, Ac, Btc, sA, sB, D, rbc, rb, w, wb, stream=stream)

        # the reference-sized workspace with the library's re-pad scratch switched off: the loader warps
        prev = lib.set_repad_scratch(0)
        cper = timed_calls(torch, lambda: cstep(ws, wsb), 10, 3, flush, stream)
        lib.set_repad_scratch(prev)
        assert lib.last_error() == lib.OK, lib.last_error_string()
        cms = sum(cper) / len(cper)
        # the same workspace as a drop-in caller has it: A re-padded into the library's scratch
        sper = timed_calls(torch, lambda: cstep(ws, wsb), 10, 3, flush, stream)
        assert lib.last_error() == lib.OK, lib.last_error_string()
        sms_ = sum(sper) / len(sper)
        # with a workspace sized for this A: re-pad into the workspace, then the tensor load
        wsa = lib.gemm_workspace_size_a(M, N, Kp, rbc)
        wsa_t = torch.empty(wsa, dtype=torch.uint8, device=dev)
        rper = timed_calls(torch, lambda: cstep(wsa_t, wsa), 10, 3, flush, stream)
        assert lib.last_error() == lib.OK, lib.last_error_string()
        rms = sum(rper) / len(rper)
        compact = {"what": f"same GEMM with A in the reference's compact layout (K={Kc}, A_row_bytes={rbc}, "
                           f"not a multiple of 32)",
                   "in_place": {"how": "workspace from the reference's query, re-pad scratch switched off "
                                       "(mxfp6_set_repad_scratch(0)): loader-warp cp.async producer",
                                "ms": cms, "tflops": 2.0 * M * N * Kc / (cms * 1e-3) / 1e12,
                                "time_ratio_vs_tensor_load": ms / cms},
                   "scratch": {"how": "workspace from the reference's query (the default): A re-padded into "
                                      "the library's stream-ordered scratch, then the tensor-load kernel",
                               "ms": sms_, "tflops": 2.0 * M * N * Kc / (sms_ * 1e-3) / 1e12,
                               "time_ratio_vs_tensor_load": ms / sms_},
                   "repad": {"how": f"workspace from gemm_workspace_size(M, N, Kp, A_row_bytes) = {wsa} bytes: "
                                    f"A re-padded into it, then the tensor-load kernel",
                             "ms": rms, "tflops": 2.0 * M * N * Kc / (rms * 1e-3) / 1e12,
                             "time_ratio_vs_tensor_load": ms / rms},
                   "device_status": lib.device_status()}
        del Ac, Btc, wsa_t
        lib.release_repad_scratch()

    # ---- the reference's own timing convention (tests/test_gemm.cpp:32-52 of eeezio/mxfp6-gemm):
    # 8 warm-ups, then 20 back-to-back calls between two events, best of 4 repetitions; no L2
    # flush between calls, so operands that fit in L2 stay there ----
    as_ref = None
    if world == 1:
        for _ in range(8):
            step()
        reps_ms = []
        for _ in range(4):
            r0 = torch.cuda.Event(enable_timing=True)
            r1 = torch.cuda.Event(enable_timing=True)
            r0.record(stream)
            for _ in range(20):
                step()
            r1.record(stream)
            torch.cuda.synchronize()
            reps_ms.append(r0.elapsed_time(r1) / 20)
        as_ref = {"ms": min(reps_ms), "tflops": 2.0 * M * N * K / (min(reps_ms) * 1e-3) / 1e12,
                  "how": "8 warm-ups, 20 back-to-back calls between events, best of 4 (no L2 flush)"}

    vs_cublas = run_vs_cublas(M, N, K, step, stream, flush, dev) if args.vs_cublas and world == 1 else None
    route = lib.route(ot, M, N, Kp)  # tile and K splits
    out_bytes = D.element_size()
    del A, sA, Bt, sB, D, ws

    # ---- BASELINE config 5 split column-parallel over the ranks (every N), other configs (N=1) ----
    strong = None
    if not args.no_strong:
        strong = strong_leg(lib, torch, dist, dev, stream, flush, rank, world, max(5, min(args.steps, 20)),
                            max(3, args.warmup), not args.no_allgather, not args.no_per_config)
    per_config = None
    if world == 1 and not args.no_per_config:
        per_config = per_config_leg(lib, torch, dev, stream, flush, max(5, min(args.steps, 20)),
                                    max(3, args.warmup), args.config)
        if strong is not None and args.config != "cfg5":
            per_config["cfg5"] = {k: v for k, v in strong.items()
                                  if k not in ("one_gpu", "efficiency_vs_one_gpu", "N_total", "N_per_gpu")}
            per_config["cfg5"]["N"] = CONFIGS["cfg5"][1]
    # ---- the reference's headline shape table, timed its way, against its published latencies ----
    ref_sweep = None
    if world == 1 and not args.no_ref_sweep:
        try:
            rows, ref_sweep = ref_sweep_leg(lib, torch, dev, stream, flush, quiet=True)
            ref_sweep["by_shape"] = [{"shape": r["shape"], "route": r["route"], "ms": r["ms"],
                                      "reference_mi350x_ms": r["reference_mi350x_ms"],
                                      "speedup": r["speedup_vs_reference"],
                                      "timed_from": "C++" if "ms_cpp" in r else "Python"} for r in rows]
        except (RuntimeError, OSError) as e:  # a failed side leg must not cost the headline line
            ref_sweep = {"error": repr(e)[:300]}

    # ---- CPU baseline (rank 0, N=1 only) ----
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        v, kind_s, cores, sample, _ = cpu_reference_sample(args.config, N, target_s=args.ref_seconds)
        cpu = {"value": v, "unit": "TFLOPS", "cores": cores, "kind": kind_s, "sample": sample}

    rf = roofline_fields(M, N, K, Kp, out_bytes, ms, wsb)
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOPS", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong" if args.strong else "weak",
            "vs_baseline": None, "dtype": "fp6_e2m3 x fp6_e2m3 -> f32 accumulate",
            "data": "synthetic (seeded E2M3 codes uniform over 64 codes, E8M0 exponents per BASELINE)",
            "config": config,
            "route": route,
            "roofline": {"bound": "tensor", "achieved": rf["tflops"], "peak": rf["peak"], "unit": "TFLOP/s",
                         "frac": rf["frac"], "traffic": NCU_TRAFFIC_BYTES.get(args.config) if world == 1 else None,
                         "algorithmic_bytes": rf["algorithmic_bytes"],
                         "peak_basis": rf["peak_basis"] + ": B200's dense FP8/FP6 tensor rate is twice bf16",
                         "best_step_ms": min(per),
                         "frac_of_nominal_fp6_dense": rf["frac_of_nominal_fp6_dense"],
                         "algorithmic_gbs": rf["algorithmic_gbs"],
                         "splitk_workspace_bytes": rf["splitk_workspace_bytes"]},  # partials written, then read
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": launches,
            "clocks": clk.summary(),
            "device_status": status,
        }
        if strong:
            line["strong"] = strong
        if per_config:
            line["per_config"] = per_config
        if ref_sweep:
            line["ref_sweep"] = ref_sweep
        if compact:
            line["compact_a"] = compact
        if as_ref:
            line["timing_as_reference"] = as_ref
        if vs_cublas:
            line["vs_cublas_mxfp8"] = vs_cublas
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


ROUTE_SWEEP_SHAPES = [(256, 256, 512, "F32"), (512, 512, 2048, "F16"), (1024, 1024, 4096, "F16"),
                      (1024, 2048, 8192, "F16"), (2048, 2048, 1024, "F16"), (2048, 2048, 4096, "F16"),
                      (512, 4096, 8192, "F16"), (4096, 1024, 4096, "F16"), (1024, 4096, 16384, "BF16"),
                      (2048, 4096, 2048, "BF16"), (4096, 4096, 4096, "F16"), (768, 3072, 4096, "BF16"),
                      (1024, 1024, 32768, "F16"), (2048, 2048, 16384, "F16")]
ROUTE_CANDIDATES = [(256, 256, 1, 0), (256, 256, 1, 1), (256, 256, 2, 0), (256, 256, 4, 0), (128, 256, 1, 0),
                    (128, 256, 2, 0), (128, 128, 1, 0), (128, 128, 2, 0), (128, 128, 4, 0)]


def run_route_sweep(reps=15):
    """Every forced route (tile, K splits, stream-K tail) on a set of shapes, L2 flushed before each
    launch, median of `reps`; one JSON line per shape with the routed choice and the fastest. The
    evidence behind the router's cost model (the operand bytes are random: timing only)."""
    sys.path.insert(0, PKG_DIR)
    import torch

    import mxfp6_b200 as lib
    torch.cuda.set_device(0)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda")
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    g = torch.Generator(device="cuda").manual_seed(SEED_A)
    for M, N, K, out in ROUTE_SWEEP_SHAPES:
        Kp = kpad(K)
        rb = Kp * 3 // 4
        A = torch.randint(0, 256, (M, rb), dtype=torch.uint8, device="cuda", generator=g)
        B = torch.randint(0, 256, (N, rb), dtype=torch.uint8, device="cuda", generator=g)
        sA = torch.randint(109, 128, (lib.tiled_scale_bytes(M, Kp),), dtype=torch.uint8, device="cuda", generator=g)
        sB = torch.randint(109, 128, (lib.tiled_scale_bytes(N, Kp),), dtype=torch.uint8, device="cuda", generator=g)
        ot = lib.OutType[out]
        D = torch.empty((M, N), dtype={"F16": torch.float16, "BF16": torch.bfloat16, "F32": torch.float32}[out],
                        device="cuda")
        wsb = max(4 * M * N * 4, lib.stream_k_bytes())
        ws = torch.empty(wsb, dtype=torch.uint8, device="cuda")
        tiles = -(-M // 256) * -(-N // 256)
        res = {}
        for MT, NT, S, sk in ROUTE_CANDIDATES:
            if S > Kp // 128 or (sk and (tiles < 74 or tiles % 74 == 0)):
                continue
            lib.gemm_force_route(ot, M, N, Kp, MT, NT, S, sk, A, B, sA, sB, D, rb, rb, ws, wsb)
            if lib.last_error() != lib.OK:
                continue
            ts = []
            for r in range(reps):
                flush.fill_(r & 0xFF)
                ev[0].record()
                lib.gemm_force_route(ot, M, N, Kp, MT, NT, S, sk, A, B, sA, sB, D, rb, rb, ws, wsb)
                ev[1].record()
                ev[1].synchronize()
                ts.append(ev[0].elapsed_time(ev[1]) * 1e3)
            res[f"{MT}x{NT}/S{S}{'/stream_k' if sk else ''}"] = round(statistics.median(ts), 2)
        if lib.device_status() != 0:
            raise RuntimeError("a kernel reported a device timeout during the route sweep")
        r = lib.route(ot, M, N, Kp)
        chosen = f"{r['MT']}x{r['NT']}/S{r['splits']}{'/stream_k' if r['stream_k'] else ''}"
        best = min(res, key=res.get)
        print(json.dumps({"shape": f"{M}x{N}x{K}", "out": out, "routed": chosen, "routed_us": res.get(chosen),
                          "fastest": best, "fastest_us": res[best], "us": res}), flush=True)
        del A, B, sA, sB, D, ws
        torch.cuda.empty_cache()


# The reference's headline sweep (benchmark_results.md:23-74 of eeezio/mxfp6-gemm): M = 2048, FP16
# output, these (N, K) shapes with the occurrence count the reference weights them by and its
# published latency on MI350X in ms (the `ours_ms` column). The rows that table marks as not
# re-measured (its former launch grid could not run them) are left out.
REF_SWEEP_M = 2048
REF_SWEEP = [
    (256, 64, 23, 0.005196), (256, 80, 22, 0.005196), (256, 96, 38, 0.005202), (256, 128, 21, 0.005200),
    (256, 144, 2, 0.005202), (256, 160, 2, 0.005192), (256, 256, 18, 0.006444), (256, 512, 1, 0.007672),
    (256, 2048, 6, 0.017478), (512, 2560, 8, 0.021470), (512, 6144, 4, 0.023780), (768, 24, 2, 0.005474),
    (768, 32, 1, 0.005464), (768, 64, 1, 0.005466), (768, 92, 1, 0.005474), (768, 96, 1, 0.005472),
    (768, 104, 1, 0.005470), (768, 152, 1, 0.005468), (768, 240, 1, 0.006770), (768, 520, 1, 0.008008),
    (768, 1840, 1, 0.016878), (1024, 1024, 10, 0.011878), (1024, 3490, 1, 0.027186),
    (1024, 12288, 20, 0.042626), (1024, 16128, 9, 0.049618), (1024, 105728, 1, 0.273237),
    (2048, 3490, 1, 0.033744), (4096, 4096, 20, 0.041052), (6144, 512, 8, 0.012954),
    (6144, 4096, 20, 0.047232), (6144, 16128, 9, 0.149118), (6144, 105728, 1, 1.040697),
    (16128, 1024, 9, 0.040318), (16384, 1024, 10, 0.043020), (20480, 6144, 9, 0.212467),
    (105728, 1024, 1, 0.293855),
]


REF_SWEEP_SETTLE_S = 1.0  # idle time before each shape (the reference runs one process per shape)
REF_SWEEP_CPP_BELOW_MS = 0.03  # rows faster than this from Python are timed again from C++


def ref_sweep_leg(lib, torch, dev, stream, flush, quiet=False):
    """The reference's headline sweep on this GPU. Each shape runs through the public entry with a
    workspace from the type-free query, as the reference's harness calls it. K is padded to kpad(K)
    with a zero tail and the FLOPs are charged at the nominal K, as the reference's table does.
    Timed the reference's way (tests/test_gemm.cpp:32-52 of eeezio/mxfp6-gemm: warm-ups, then 20
    back-to-back calls between two events, best of 4) and, for comparison, L2-flushed single
    calls (median of 10). The reference times each shape in a process of its own from C++ with its
    clocks locked; here the GPU idles REF_SWEEP_SETTLE_S before each shape (its clocks are not
    locked: the 1 kW cap sets them under load, and the NVML median is reported per row), and rows
    short enough for Python's per-call enqueue cost to show are timed again from the C++ drop-in
    caller (same convention, its own process), whose figure is the row's `ms`. Returns per-shape
    rows and a summary against the published MI350X latencies. Operand codes are random bytes
    (uniform over the 64 codes; timing only)."""
    import subprocess
    import tempfile
    M = REF_SWEEP_M
    ot = lib.OutType.F16
    g = torch.Generator(device=dev).manual_seed(SEED_A + 7)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    rows = []
    tmp = tempfile.TemporaryDirectory()
    try:
        exe = build_cpp_caller(tmp.name)
    except (OSError, subprocess.SubprocessError):
        exe = None
    for N, K, count, ref_ms in REF_SWEEP:
        time.sleep(REF_SWEEP_SETTLE_S)
        Kp = kpad(K)
        rb = Kp * 3 // 4
        used = K * 3 // 4
        A = torch.randint(0, 256, (M, rb), dtype=torch.uint8, device=dev, generator=g)
        Bt = torch.randint(0, 256, (N, rb), dtype=torch.uint8, device=dev, generator=g)
        A[:, used:] = 0
        Bt[:, used:] = 0
        sA = torch.randint(118, 128, (lib.tiled_scale_bytes(M, Kp),), dtype=torch.uint8, device=dev, generator=g)
        sB = torch.randint(118, 128, (lib.tiled_scale_bytes(N, Kp),), dtype=torch.uint8, device=dev, generator=g)
        D = torch.empty((M, N), dtype=torch.float16, device=dev)
        wsb = lib.gemm_workspace_size(M, N, Kp)
        ws = torch.empty(wsb, dtype=torch.uint8, device=dev) if wsb else None

        def call():
            lib.gemm(ot, M, N, Kp, A, Bt, sA, sB, D, rb, rb, ws, wsb, stream=stream)

        for _ in range(8):
            call()
        torch.cuda.synchronize()
        best = float("inf")
        with ClockSampler(dev.index if isinstance(dev, torch.device) and dev.index is not None else 0) as clk:
            for _ in range(4):
                ev[0].record(stream)
                for _ in range(20):
                    call()
                ev[1].record(stream)
                ev[1].synchronize()
                best = min(best, ev[0].elapsed_time(ev[1]) / 20)
        single = []
        for r in range(10):
            flush.fill_(r & 0xFF)
            ev[0].record(stream)
            call()
            ev[1].record(stream)
            ev[1].synchronize()
            single.append(ev[0].elapsed_time(ev[1]))
        if lib.last_error() != lib.OK or lib.device_status() != 0:
            raise RuntimeError(f"reference sweep 2048x{N}x{K}: error {lib.last_error()}")
        r = lib.route(ot, M, N, Kp)
        row = {"shape": f"{M}x{N}x{K}", "count": count,
               "route": f"{r['MT']}x{r['NT']}/S{r['splits']}" + ("/stream_k" if r["stream_k"] else "")
                        + ("/banded" if r["banded"] else ""),
               "ms_python": best, "ms_l2_flushed": statistics.median(single), "clocks": clk.summary()}
        ms = best
        if exe and best < REF_SWEEP_CPP_BELOW_MS:
            time.sleep(REF_SWEEP_SETTLE_S)
            row["ms_cpp"] = ms = cpp_time(exe, (M, N, K, "F16")) * 1e-3
        row.update({"ms": ms, "tflops": 2.0 * M * N * K / (ms * 1e-3) / 1e12, "reference_mi350x_ms": ref_ms,
                    "speedup_vs_reference": ref_ms / ms})
        rows.append(row)
        if not quiet:
            print(json.dumps(row), flush=True)
        del A, Bt, sA, sB, D, ws
    torch.cuda.empty_cache()
    tmp.cleanup()
    sp = [r["speedup_vs_reference"] for r in rows]
    ours_w = sum(r["count"] * r["ms"] for r in rows)
    ref_w = sum(r["count"] * r["reference_mi350x_ms"] for r in rows)
    worst = min(rows, key=lambda r: r["speedup_vs_reference"])
    return rows, {"what": "the reference's headline sweep (M=2048, FP16 out, its (N, K) list), timed its way "
                          "(best of 4 x 20 back-to-back calls), against its published MI350X latencies",
                  "rows": len(rows), "count_weighted_ms": ours_w, "reference_count_weighted_ms": ref_w,
                  "count_weighted_speedup": ref_w / ours_w,
                  "geomean_speedup": math.exp(sum(math.log(x) for x in sp) / len(sp)),
                  "min_speedup": {"shape": worst["shape"], "speedup": worst["speedup_vs_reference"]},
                  "rows_below_1": sum(1 for x in sp if x < 1.0)}


def run_ref_sweep():
    sys.path.insert(0, PKG_DIR)
    import torch

    import mxfp6_b200 as lib
    torch.cuda.set_device(0)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda")
    _, summary = ref_sweep_leg(lib, torch, "cuda", torch.cuda.current_stream(), flush)
    print(json.dumps({"summary": summary}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="cfg2")
    ap.add_argument("--shape", default=None,
                    help="MxNxK:OUT (OUT F32/F16/BF16): time this shape instead of a BASELINE config (E2M3 codes "
                         "uniform over the 64 codes, E8M0 exponents in [109, 127]); for profiling one route")
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end leg")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-allgather", action="store_true", help="skip the gathers of the config-5 D shards")
    ap.add_argument("--no-strong", action="store_true", help="skip the config-5 column-split leg")
    ap.add_argument("--no-per-config", action="store_true", help="skip the other BASELINE configs (N=1)")
    ap.add_argument("--with-compact", action="store_true",
                    help="also time the same GEMM with A in the reference's compact layout (loader warps, "
                         "library re-pad scratch, caller workspace)")
    ap.add_argument("--ref-seconds", type=float, default=10.0, help="target CPU seconds per reference sample")
    ap.add_argument("--e2e-cols", type=int, default=2,
                    help="column chunks of B and D in the end-to-end pipeline (1 = row chunks only)")
    ap.add_argument("--e2e-rows", type=int, default=E2E_ROW_CHUNKS,
                    help="row chunks of A and D in the end-to-end pipeline (1 = column chunks only)")
    ap.add_argument("--strong", action="store_true",
                    help="split the config's N over the ranks (strong scaling) instead of N per rank")
    ap.add_argument("--shard-of", type=int, default=1,
                    help="on one GPU, run the N shard one rank of this many holds (strong scaling)")
    ap.add_argument("--import-only", action="store_true",
                    help="only time the device import of the config's B from the reference's layout")
    ap.add_argument("--no-ref-sweep", action="store_true",
                    help="skip the reference's headline shape table in the N=1 line")
    ap.add_argument("--ref-sweep", action="store_true",
                    help="time the reference's headline shape sweep (M=2048, FP16) and compare with its "
                         "published MI350X latencies; one JSON line per shape and a summary")
    ap.add_argument("--route-sweep", action="store_true",
                    help="time every forced route on a set of shapes (L2 flushed) next to the routed choice")
    ap.add_argument("--vs-cublas", action="store_true",
                    help="also time cuBLASLt's MXFP8 block-scaled GEMM on the same shape (interleaved "
                         "with this library's, then each sustained for about a second with clocks)")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    if args.shape:
        dims, out = args.shape.split(":")
        M, N, K = (int(x) for x in dims.lower().split("x"))
        CONFIGS["shape"] = (M, N, K, "codes", (109, 127), out.upper())
        CONFIG_DESC["shape"] = f"MXFP6 GEMM M={M} N={N} K={K}, {out.upper()} output"
        args.config = "shape"
    if args.ref_sweep:
        run_ref_sweep()
    elif args.route_sweep:
        run_route_sweep()
    elif args.import_only:
        sys.path.insert(0, PKG_DIR)
        import torch

        import mxfp6_b200 as lib
        M, N, K = CONFIGS[args.config][:3]
        rb = lib.kpad(K) * 3 // 4
        dev = torch.device("cuda", 0)
        print(json.dumps({"import_ref_B_device": time_import_leg(lib, N, K, rb, torch.cuda.current_stream(dev), dev)}))
    elif args.impl == "reference":
        run_reference_arm(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
