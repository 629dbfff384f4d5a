#!/usr/bin/env python3
"""Benchmark of the batched C2C FFT hot path and of the
2-D FFT convolution (``--workload conv2d``).

Default workload (one "step"): forward then unnormalized inverse C2C FFT,
N = 1024, batch 65536 per GPU, float2 storage / TF32 tensor-core arithmetic,
separate input/output buffers, re/im i.i.d. U[-1,1) from a seed (synthetic:
the reference publishes no dataset).  Each buffer is 512 MiB, larger than the
126 MB L2, so every launch streams from HBM.

Metric: HBM throughput of the transform in GB/s (algorithmic bytes: read N*8 +
write N*8 per transform, twiddles excluded) — the reference's metric is
"batched C2C FFT us & HBM GB/s (% peak)".  `value` is the whole-job aggregate
over all ranks (weak scaling: every rank transforms its own 65536 signals;
the batch dimension shards with no collective on the data path).

``--workload conv2d``: one step = one circular 2-D convolution call over the
rank's images of config 5 (64 x 32 real fp32 512x512 images, one 31x31
filter per channel).  ``--scaling strong`` (default) splits the 64 batch
images by image pair across the ranks; ``weak`` gives every rank all 2048.
Metric: GB/s of algorithmic bytes (read 4 + write 4 bytes per pixel).

Usage:  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                        [--workload c2c|conv2d] [--scaling strong|weak]
Under torchrun each rank uses LOCAL_RANK's GPU; rank 0 prints one JSON line.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

N = 1024
BATCH = 65536
ESZ = 8  # float2
BYTES_PER_TRANSFORM_BATCH = 2 * N * BATCH * ESZ          # read + write, one direction
METRIC = "batched C2C FFT HBM GB/s (N=1024, batch 65536/GPU, TF32 fwd+inv)"
DTYPE = "float"

# BASELINE config 5
CONV2D_B, CONV2D_C, CONV2D_HW, CONV2D_F = 64, 32, 512, 31
CONV2D_METRIC = "2-D FFT convolution HBM GB/s (config 5: 64x32 fp32 512x512 images, 31x31 per channel)"


def configure(n: int, batch: int, dtype: str) -> None:
    """Non-default workloads (profiling / sweeps); the default is config 2."""
    global N, BATCH, ESZ, BYTES_PER_TRANSFORM_BATCH, METRIC, DTYPE
    N, BATCH, DTYPE = n, batch, dtype
    ESZ = 8 if dtype == "float" else 4
    BYTES_PER_TRANSFORM_BATCH = 2 * N * BATCH * ESZ
    prec = "TF32" if dtype == "float" else "FP16"
    METRIC = f"batched C2C FFT HBM GB/s (N={N}, batch {BATCH}/GPU, {prec} fwd+inv)"


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return float(d["hbm_gbs"]), "measured"
        except Exception:
            pass
    return 6650.0, "fallback"


def profile_value(name: str, key: str):
    """An integer `key: <int>` line from a committed ncu summary under
    profiles/, else None."""
    p = ROOT / "profiles" / name
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.strip().startswith(key + ":"):
            try:
                return int(line.split(":", 1)[1].strip().split()[0])
            except ValueError:
                return None
    return None


class ClockSampler:
    """SM clock and clock-event reasons of one GPU, read through NVML every
    10 ms on a background thread while the timed region runs (reading only;
    no setting is changed)."""

    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
               0x4: "sw_power_cap", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, cuda_index: int, period_s: float = 0.01):
        self.cuda_index = cuda_index
        self.period = period_s
        self.samples = []
        self.extra = []          # (memory MHz, power W, GPU temperature C) per sample
        self.max_mhz = None
        self.error = None
        self._stop = threading.Event()
        self._t = None
        self._nvml = None
        self._h = None

    def _handle(self):
        import pynvml
        import torch

        pynvml.nvmlInit()
        props = torch.cuda.get_device_properties(self.cuda_index)
        uuid = str(getattr(props, "uuid", "") or "")
        if uuid:
            try:
                return pynvml, pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
            except Exception:
                pass
        try:
            bus = f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"
            return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.cuda_index)

    def __enter__(self):
        try:
            self._nvml, self._h = self._handle()
            self.max_mhz = float(self._nvml.nvmlDeviceGetMaxClockInfo(self._h, self._nvml.NVML_CLOCK_SM))
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        except Exception as e:  # NVML unavailable: the line says so
            self.error = f"{type(e).__name__}: {e}"
        return self

    def _reasons(self):
        f = getattr(self._nvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            self._nvml.nvmlDeviceGetCurrentClocksThrottleReasons
        return int(f(self._h))

    def _run(self):
        nv = self._nvml
        while not self._stop.is_set():
            try:
                mhz = float(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                self.samples.append((mhz, self._reasons()))
                self.extra.append((float(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_MEM)),
                                   float(nv.nvmlDeviceGetPowerUsage(self._h)) / 1000.0,
                                   float(nv.nvmlDeviceGetTemperature(self._h, nv.NVML_TEMPERATURE_GPU))))
            except Exception as e:
                self.error = f"{type(e).__name__}: {e}"
                return
            self._stop.wait(self.period)

    def __exit__(self, *exc):
        self._stop.set()
        if self._t is not None:
            self._t.join(timeout=2)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0,
                    "source": "nvml", "error": self.error}
        reasons = set()
        for _, r in self.samples:
            for bit, name in self.REASONS.items():
                if r & bit:
                    reasons.add(name)
        out = {"sm_mhz": statistics.median(m for m, _ in self.samples), "sm_max_mhz": self.max_mhz,
               "reasons": sorted(reasons), "samples": len(self.samples), "source": "nvml, 10 ms, timed region"}
        if self.extra:
            out["mem_mhz"] = statistics.median(e[0] for e in self.extra)
            out["power_w_median"] = statistics.median(e[1] for e in self.extra)
            out["power_w_max"] = max(e[1] for e in self.extra)
            out["temp_c_first_last"] = [self.extra[0][2], self.extra[-1][2]]
        return out


class CuFFT:
    """cuFFT on the same GPU as an extra comparison point (the reference's
    baseline is sample/bench/baseline/baseline_cufft.cu:28-69): one batched
    1-D C2C plan, cufftMakePlanMany (complex64) or cufftXtMakePlanMany with
    CUDA_C_16F (half2), executed with cufftExecC2C / cufftXtExec on the
    bench's stream.  Uses the libcufft that torch has already loaded."""

    C2C, FORWARD, INVERSE = 0x29, -1, 1
    CUDA_C_16F, CUDA_C_32F = 6, 4

    def __init__(self, n: int, batch: int, half: bool, stream: int):
        lib = ctypes.CDLL("libcufft.so.11")
        self.lib, self.half = lib, half
        self.h = ctypes.c_int(0)
        self._ok(lib.cufftCreate(ctypes.byref(self.h)), "cufftCreate")
        ws = ctypes.c_size_t(0)
        if half:
            nn = (ctypes.c_longlong * 1)(n)
            lib.cufftXtMakePlanMany.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                                                ctypes.c_longlong, ctypes.c_longlong, ctypes.c_int, ctypes.c_void_p,
                                                ctypes.c_longlong, ctypes.c_longlong, ctypes.c_int, ctypes.c_longlong,
                                                ctypes.c_void_p, ctypes.c_int]
            self._ok(lib.cufftXtMakePlanMany(self.h, 1, nn, None, 1, n, self.CUDA_C_16F, None, 1, n, self.CUDA_C_16F,
                                             batch, ctypes.byref(ws), self.CUDA_C_16F), "cufftXtMakePlanMany")
        else:
            nn = (ctypes.c_int * 1)(n)
            lib.cufftMakePlanMany.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                                              ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                              ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
            self._ok(lib.cufftMakePlanMany(self.h, 1, nn, None, 1, n, None, 1, n, self.C2C, batch, ctypes.byref(ws)),
                     "cufftMakePlanMany")
        lib.cufftSetStream.argtypes = [ctypes.c_int, ctypes.c_void_p]
        self._ok(lib.cufftSetStream(self.h, ctypes.c_void_p(stream)), "cufftSetStream")
        self.workspace_bytes = int(ws.value)

    @staticmethod
    def _ok(rc, what):
        if rc != 0:
            raise RuntimeError(f"{what} failed with cuFFT status {rc}")

    def __call__(self, x_ptr: int, y_ptr: int, forward: bool):
        d = self.FORWARD if forward else self.INVERSE
        if self.half:
            self._ok(self.lib.cufftXtExec(self.h, ctypes.c_void_p(x_ptr), ctypes.c_void_p(y_ptr), d), "cufftXtExec")
        else:
            self._ok(self.lib.cufftExecC2C(self.h, ctypes.c_void_p(x_ptr), ctypes.c_void_p(y_ptr), d), "cufftExecC2C")

    def close(self):
        if self.h.value:
            self.lib.cufftDestroy(self.h)
            self.h = ctypes.c_int(0)


def cpu_baseline(seconds: float = 12.0, sample_batch: int = 0):
    """FP64 oracle FFT (fwd + inv) on the host cores over a bounded sample of
    the same workload (a quarter of the per-GPU batch, as in the reference
    arm); reported in the metric's unit (GB/s of algorithmic bytes).  TEST
    INFRASTRUCTURE: the oracle is the checker/baseline only."""
    import oracle

    sample_batch = sample_batch or max(1, BATCH // 4)
    threads = oracle.hardware_threads()
    rng = np.random.default_rng(7)
    x = (rng.uniform(-1, 1, (sample_batch, N)) + 1j * rng.uniform(-1, 1, (sample_batch, N))).astype(np.complex64)
    oracle.fft_f32io(x[:16], True, threads)
    t0 = time.perf_counter()
    reps = 0
    while True:
        y = oracle.fft_f32io(x, True, threads)
        oracle.fft_f32io(y, False, threads)
        reps += 1
        if time.perf_counter() - t0 >= seconds:
            break
    dt = time.perf_counter() - t0
    bytes_done = reps * 2 * (2 * N * sample_batch * ESZ)
    return {"value": bytes_done / dt / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{reps} x (fwd+inv) of {sample_batch} signals of N={N} (FP64 radix-2, float2 I/O), "
                      f"{dt:.1f} s on {threads} threads"}


def conv2d_cpu_sample(seconds: float = 10.0):
    """FP64 direct circular 2-D convolution (the oracle's restatement of the
    reference's host-side convolution check, conv2d/main.cu:42-125, made
    circular as config 5 defines it) over a bounded sample of config-5
    images, all host threads.  Returns (GB/s of algorithmic bytes, images,
    seconds, threads).  TEST INFRASTRUCTURE: the baseline only."""
    import oracle

    threads = oracle.hardware_threads()
    hw, f = CONV2D_HW, CONV2D_F
    rng = np.random.default_rng(11)
    x = rng.standard_normal((threads, hw, hw))
    filt = rng.standard_normal((CONV2D_C, f, f))
    idx = (np.arange(threads) % CONV2D_C).astype(np.int32)
    oracle.circconv2d(x[:1, :64, :64].copy(), filt[:, :5, :5].copy(), idx[:1], threads)
    t0 = time.perf_counter()
    images = 0
    while True:
        oracle.circconv2d(x, filt, idx, threads)
        images += threads
        if time.perf_counter() - t0 >= seconds:
            break
    dt = time.perf_counter() - t0
    return images * hw * hw * 8 / dt / 1e9, images, dt, threads


SWEEP_N = (64, 128, 256, 512, 1024, 2048, 4096)


def run_sweep(args):
    """Per-size table (not the contract line): every N and storage type in both
    directions at BASELINE config 3's batch 2^26/N (divided by --sweep-scale),
    plus config 3's masked partial batch (batch - 7) for half2, with cuFFT on
    the same buffers beside each full batch, then the conv1d (config 4),
    conv2d (config 5) and tiled conv1d kernels.  Event-timed on one GPU,
    inputs resident in HBM, each launch streaming buffers larger than L2 at
    scale 1.  Prints a markdown table."""
    import torch
    import thunderfft_b200 as tf

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev)
    peak, peak_kind = measured_peaks()
    steps, warm = max(args.steps, 1), args.warmup

    def timed(fn):
        for _ in range(warm):
            fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        tf.sync_check(stream)
        return e0.elapsed_time(e1) / steps * 1e3  # us per call

    print(f"| storage | N | batch | direction | us / launch | transforms/s | GB/s | of {peak_kind} peak "
          f"({peak:.0f} GB/s) | rel. L2 (round trip) | cuFFT us | cuFFT GB/s |")
    print("|---|---|---|---|---|---|---|---|---|---|---|")
    g = torch.Generator(device=dev)
    g.manual_seed(33)
    only = args.sweep_only
    for dtype in (("float", "half") if only in ("all", "fft") else ()):
        esz = 8 if dtype == "float" else 4
        for n in SWEEP_N:
            full = (1 << 26) // n // args.sweep_scale
            for b in ((full, full - 7) if dtype == "half" else (full,)):
                if dtype == "float":
                    x = torch.complex(torch.rand(b, n, device=dev, generator=g) * 2 - 1,
                                      torch.rand(b, n, device=dev, generator=g) * 2 - 1).contiguous()
                else:
                    x = (torch.rand(b, n, 2, device=dev, generator=g) - 0.5).half()
                y, z = torch.empty_like(x), torch.empty_like(x)
                tf.ThunderFFTInitialize(dtype, n)
                us_f = timed(lambda: tf.c2c_async(dtype, n, True, x, y, b, stream))
                us_i = timed(lambda: tf.c2c_async(dtype, n, False, y, z, b, stream))
                xs = torch.view_as_real(x[:256]) if x.is_complex() else x[:256].float()
                zs = torch.view_as_real(z[:256]) if z.is_complex() else z[:256].float()
                err = float(((zs / n - xs).pow(2).sum() / xs.pow(2).sum()).sqrt())
                cu = {"fwd": None, "inv": None}
                if b == full and not args.no_cufft:
                    try:
                        plan = CuFFT(n, b, dtype == "half", stream.cuda_stream)
                        cu["fwd"] = timed(lambda: plan(x.data_ptr(), y.data_ptr(), True))
                        cu["inv"] = timed(lambda: plan(y.data_ptr(), z.data_ptr(), False))
                        plan.close()
                    except Exception as e:  # pragma: no cover
                        print(f"<!-- cuFFT N={n} {dtype}: {e} -->")
                for d, us in (("fwd", us_f), ("inv", us_i)):
                    gbs = 2 * n * b * esz / us / 1e3
                    cus = cu[d]
                    cu_cols = (f"{cus:.1f} | {2 * n * b * esz / cus / 1e3:.0f}" if cus else "— | —")
                    print(f"| {'float2' if dtype == 'float' else 'half2'} | {n} | {b} | {d} | {us:.1f} | "
                          f"{b / us * 1e6:.3e} | {gbs:.0f} | {gbs / peak:.3f} | {err:.2e} | {cu_cols} |", flush=True)
                del x, y, z
                torch.cuda.empty_cache()
    if args.no_conv or only == "fft":
        return 0
    if only in ("all", "conv1d"):
        sweep_conv1d(args, tf, dev, g, stream, timed, peak)
    if only in ("all", "conv2d"):
        sweep_conv2d(args, tf, dev, g, stream, timed, peak)
    if only in ("all", "tiled"):
        sweep_tiled(args, tf, dev, g, stream, timed, peak)
    return 0


def sweep_tiled(args, tf, dev, g, stream, timed, peak):
    """Tiled (overlap-save) conv1d row: the reference sample's shape
    (sample/conv1d/main.cu: one half2 sequence, 9 taps by default,
    --tiled-taps), 2^24 elements / --sweep-scale.  Bandwidth counts the sequence read once and the valid
    outputs written once."""
    import torch

    L, taps = (1 << 24) // args.sweep_scale, args.tiled_taps
    x = (torch.rand(1, L, 2, device=dev, generator=g) - 0.5).half()
    filt = torch.complex(torch.rand(taps, device=dev, generator=g) - 0.5,
                         torch.rand(taps, device=dev, generator=g) - 0.5).contiguous()
    op = tf.conv1d_tiled_operator(filt, "half")
    y = torch.empty(1, L - taps + 1, 2, dtype=torch.float16, device=dev)
    us = timed(lambda: tf.conv1d_tiled(x, op, taps, out=y, stream=stream, sync=False))
    alg = (L + (L - taps + 1)) * 4
    print(f"| tiled conv1d half2, {taps} taps | 64 | 1 x {L} | windows*H | {us:.1f} | — | {alg / us / 1e3:.0f} | "
          f"{alg / us / 1e3 / peak:.3f} | | | |", flush=True)


def sweep_conv1d(args, tf, dev, g, stream, timed, peak):
    """conv1d row of the sweep: BASELINE config 4 (batch / --sweep-scale)."""
    import torch

    tf.conv1d_set_arithmetic(args.conv_arith)
    B1, lin, taps, n1 = 16384 // args.sweep_scale, 3072, 1025, 4096
    xs = torch.randn(B1, lin, device=dev, generator=g)
    hs = torch.randn(taps, device=dev, generator=g)
    spec = tf.conv1d_filter_spectrum(hs, n1)
    ys = torch.empty(B1, n1, device=dev)
    us = timed(lambda: tf.conv1d(xs, spec, n1, out=ys, stream=stream, sync=False))
    alg = B1 * (lin + n1) * 4
    print(f"| conv1d fp32 (config 4), {args.conv_arith} | {n1} | {B1} x {lin} | fwd*H*inv | {us:.1f} | "
          f"{B1 / us * 1e6:.3e} | {alg / us / 1e3:.0f} | {alg / us / 1e3 / peak:.3f} | | | |", flush=True)


def sweep_conv2d(args, tf, dev, g, stream, timed, peak):
    """conv2d row of the sweep: BASELINE config 5 (batch / --sweep-scale)."""
    import torch

    tf.conv2d_set_arithmetic(args.conv_arith)
    B2, C2, hw, f = CONV2D_B // args.sweep_scale, CONV2D_C, CONV2D_HW, CONV2D_F
    xi = torch.randn(B2, C2, hw, hw, device=dev, generator=g)
    fi = torch.randn(C2, f, f, device=dev, generator=g)
    sp = tf.conv2d_filter_spectra(fi, hw, hw)
    ws = tf.conv2d_workspace(hw, hw, (B2 // 2) * C2)
    yi = torch.empty_like(xi)
    us = timed(lambda: tf.conv2d(xi, sp, ws, out=yi, stream=stream, sync=False))
    alg = 2 * xi.numel() * 4
    print(f"| conv2d fp32 (config 5), {args.conv_arith} | {hw}x{hw} | {B2} x {C2} | fwd*H*inv | {us:.1f} | "
          f"{B2 * C2 / us * 1e6:.3e} images | {alg / us / 1e3:.0f} | {alg / us / 1e3 / peak:.3f} | | | |", flush=True)


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def run_reference(args):
    """Reference arm: the reference's CPU path for this workload.  The
    reference has no host FFT (its checker is cuFFT); the arm times the FP64
    CPU restatement on all host threads, rank 0 only.  For conv2d it times
    the FP64 direct circular convolution on a bounded sample of images."""
    world, rank, _ = dist_setup()
    if rank != 0:
        return 0
    import oracle

    threads = oracle.hardware_threads()
    if args.workload == "conv2d":
        for _ in range(args.warmup):
            conv2d_cpu_sample(0.0)
        t0 = time.perf_counter()
        images = 0
        for _ in range(args.steps):
            images += conv2d_cpu_sample(0.0)[1]
        dt = time.perf_counter() - t0
        value = images * CONV2D_HW * CONV2D_HW * 8 / dt / 1e9
        total = CONV2D_B * CONV2D_C
        line = {
            "impl": "reference", "metric": CONV2D_METRIC, "value": value, "unit": "GB/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / images * total * 1e3,
            "higher_is_better": True, "scaling": args.scaling, "vs_baseline": None, "dtype": "f64",
            "data": "synthetic",
            "config": {"workload": f"conv2d config 5 ({total} images; bounded CPU sample of {threads} images "
                                   "per step)", "images": total, "hw": CONV2D_HW, "filter": CONV2D_F},
            "cpu_baseline": {"value": value, "unit": "GB/s", "cores": threads, "kind": "port",
                             "sample": f"{args.steps} steps x {threads} images, FP64 direct circular convolution"},
            "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }
        print(json.dumps(line), flush=True)
        return 0
    # a quarter of the per-GPU batch per step: tens of milliseconds of CPU
    # work, so thread start-up and clock ramp do not dominate a short run
    sample_batch = max(1, BATCH // 4)
    rng = np.random.default_rng(7)
    x = (rng.uniform(-1, 1, (sample_batch, N)) + 1j * rng.uniform(-1, 1, (sample_batch, N))).astype(np.complex64)
    for _ in range(args.warmup):
        oracle.fft_f32io(oracle.fft_f32io(x, True, threads), False, threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oracle.fft_f32io(oracle.fft_f32io(x, True, threads), False, threads)
    dt = time.perf_counter() - t0
    value = args.steps * 2 * (2 * N * sample_batch * ESZ) / dt / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3 * (BATCH / sample_batch),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": {"workload": f"C2C fwd+inv, N={N}, batch {BATCH} per GPU (bounded CPU sample of {sample_batch} signals)",
                   "n": N, "batch_per_gpu": BATCH, "storage": "float2"},
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"{args.steps} steps x (fwd+inv) of {sample_batch} signals, FP64 oracle"},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "transforms_per_s": args.steps * 2 * sample_batch / dt,
    }
    print(json.dumps(line), flush=True)
    return 0


class Ranks:
    """One process per GPU (torchrun env), NCCL only for barriers and the
    max-over-ranks timing reduction."""

    def __init__(self):
        import torch

        self.world, self.rank, self.local = dist_setup()
        torch.cuda.set_device(self.local)
        self.dev = torch.device("cuda", self.local)
        self.dist = None
        if self.world > 1:
            import datetime
            import torch.distributed as dist_mod

            dist_mod.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=self.dev)
            self.dist = dist_mod

    def barrier(self):
        if self.dist is not None:
            self.dist.barrier()

    def max(self, v: float) -> float:
        import torch

        t = torch.tensor([v], device=self.dev, dtype=torch.float64)
        if self.dist is not None:
            self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def max_each(self, values):
        """Elementwise max over ranks of a list of equal length on every rank."""
        import torch

        t = torch.tensor(values, device=self.dev, dtype=torch.float64)
        if self.dist is not None:
            self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return [float(v) for v in t.tolist()]

    def agree(self, flag: bool) -> bool:
        """Rank 0's flag, on every rank."""
        import torch

        if self.dist is None:
            return flag
        t = torch.tensor([1 if flag else 0], device=self.dev, dtype=torch.int32)
        self.dist.broadcast(t, src=0)
        return bool(t.item())

    def close(self):
        if self.dist is not None:
            self.dist.barrier()
            self.dist.destroy_process_group()


def timed_region(ranks, stream, steps, step, tf, min_seconds: float = 0.25):
    """The timed region, repeated: each repeat is exactly K steps, bracketed
    by a barrier and a device synchronize on both sides, and event-timed on
    `stream`.  It repeats at least 5 times and until `min_seconds` have
    passed (at most 200 times), with the NVML clock sampler running
    throughout, so that the clock record describes the timed steps even when
    K steps take only milliseconds.  Each repeat's time is the max over
    ranks; the result is their median.  Returns (median ms, per-repeat ms,
    library kernel launches per repeat, clock summary)."""
    import torch

    per_rank = []
    launches = None
    with ClockSampler(ranks.local) as clocks:
        t0 = time.perf_counter()
        while len(per_rank) < 200:
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ranks.barrier()
            torch.cuda.synchronize(ranks.dev)
            l0 = tf.launch_count()
            ev0.record(stream)
            for _ in range(steps):
                step()
            ev1.record(stream)
            if launches is None:
                launches = tf.launch_count() - l0
            torch.cuda.synchronize(ranks.dev)
            ranks.barrier()
            per_rank.append(ev0.elapsed_time(ev1))
            # every rank takes the same number of repeats: rank 0 decides
            done = len(per_rank) >= 5 and time.perf_counter() - t0 >= min_seconds
            if not ranks.agree(done):
                continue
            break
    tf.sync_check(stream)
    reps = ranks.max_each(per_rank)
    return statistics.median(reps), reps, launches, clocks.summary()


def run_c2c(args):
    import torch
    import thunderfft_b200 as tf
    from thunderfft_b200.shard import weak_scaling_value

    ranks = Ranks()
    world, rank, dev = ranks.world, ranks.rank, ranks.dev
    stream = torch.cuda.current_stream(dev)
    g = torch.Generator(device=dev)
    g.manual_seed(1234 + rank)
    if DTYPE == "float":
        x = torch.complex(torch.rand(BATCH, N, device=dev, generator=g) * 2 - 1,
                          torch.rand(BATCH, N, device=dev, generator=g) * 2 - 1).contiguous()
    else:
        x = (torch.rand(BATCH, N, 2, device=dev, generator=g) - 0.5).half()
    y = torch.empty_like(x)
    z = torch.empty_like(x)
    tf.ThunderFFTInitialize(DTYPE, N)

    def step():
        tf.c2c_async(DTYPE, N, True, x, y, BATCH, stream)
        tf.c2c_async(DTYPE, N, False, y, z, BATCH, stream)

    for _ in range(max(args.warmup, 3)):
        step()
    tf.sync_check(stream)

    # correctness gate on a slice of this very run (round trip / N)
    def _planes(t):  # (re, im) pairs as float32 for either storage type
        return torch.view_as_real(t).float() if t.is_complex() else t.float()

    xs, zs = _planes(x[:64]), _planes(z[:64])
    rt_err = float(((zs / N - xs).abs().pow(2).sum() / xs.abs().pow(2).sum()).sqrt())
    if not rt_err <= 5e-3:  # the reference's gate (also catches NaN)
        raise RuntimeError(f"round trip rel-L2 {rt_err} fails the 5e-3 gate")

    # ---- device-timed region (inputs resident in HBM, buffers > L2)
    ms_max, reps, launches, clocks = timed_region(ranks, stream, args.steps, step, tf)
    ms_per_step = ms_max / args.steps
    value = weak_scaling_value(args.steps * 2 * BYTES_PER_TRANSFORM_BATCH, ms_max, world)
    per_launch_us = ms_max / (2 * args.steps) * 1e3
    achieved = BYTES_PER_TRANSFORM_BATCH / (per_launch_us / 1e6) / 1e9

    # ---- cuFFT on the same GPU / same buffers (extra comparison point)
    cufft = None
    if not args.no_extras:
        try:
            plan = CuFFT(N, BATCH, DTYPE == "half", stream.cuda_stream)
            for _ in range(3):
                plan(x.data_ptr(), y.data_ptr(), True)
                plan(y.data_ptr(), z.data_ptr(), False)
            torch.cuda.synchronize(dev)
            c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            cu_reps = 50
            c0.record(stream)
            for _ in range(cu_reps):
                plan(x.data_ptr(), y.data_ptr(), True)
                plan(y.data_ptr(), z.data_ptr(), False)
            c1.record(stream)
            torch.cuda.synchronize(dev)
            plan.close()
            cms = c0.elapsed_time(c1) / cu_reps
            cufft = {"value": 2 * BYTES_PER_TRANSFORM_BATCH / (cms / 1e3) / 1e9, "unit": "GB/s", "ms_per_step": cms,
                     "what": (f"cuFFT {'cufftXtExec CUDA_C_16F' if DTYPE == 'half' else 'cufftExecC2C'} "
                              f"(cufft{'Xt' if DTYPE == 'half' else ''}MakePlanMany, batch {BATCH}) fwd+inv, "
                              "same buffers, 1 GPU"),
                     "plan_workspace_bytes": plan.workspace_bytes}
        except Exception as e:  # pragma: no cover
            cufft = {"error": str(e)}

    # ---- end to end through the public API with host buffers
    e2e = None
    if not args.no_extras:
        try:
            e2e = c2c_end_to_end(ranks, stream, x, tf)
        except Exception as e:  # pragma: no cover
            e2e = {"error": str(e)}

    peak, peak_kind = measured_peaks()
    if rank == 0:
        cpu = None if args.no_cpu_baseline or world > 1 else cpu_baseline()
        line = {
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": max(args.warmup, 3), "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "tf32" if DTYPE == "float" else "f16",
            "data": "synthetic",
            "config": {"workload": (f"C2C fwd+inv (BASELINE config 2), N={N}, batch {BATCH} per GPU, float2"
                                    if DTYPE == "float" else f"C2C fwd+inv FP16, N={N}, batch {BATCH} per GPU"),
                       "n": N, "batch_per_gpu": BATCH, "storage": "float2" if DTYPE == "float" else "half2",
                       "parallelism": f"batch-shard x{world}, no collective",
                       "l2": (f"inputs {N * BATCH * ESZ >> 20} MiB per buffer > 126 MB L2 (no flush needed)"
                              if N * BATCH * ESZ > 126e6 else "WARNING: buffers fit in L2")},
            "us_per_transform_batch": per_launch_us,
            "transforms_per_s": world * args.steps * 2 * BATCH / (ms_max / 1e3),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak,
                         "traffic": profile_value("fft2_f32_n1024_b65536.md", "traffic_bytes_per_launch"),
                         "kernel": (f"thff::fft2_kernel<Fft2Cfg<{str(DTYPE == 'half').lower()},{N}>>" if N > 64
                                    else f"thff::dft1_kernel<Dft1Cfg<{str(DTYPE == 'half').lower()}>>"),
                         "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                         else "fallback 6650 GB/s"},
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": launches,
            "timing": {"repeats": len(reps), "steps_per_repeat": args.steps,
                       "ms_min": min(reps), "ms_median": ms_max, "ms_max": max(reps),
                       "ms_each": [round(v, 4) for v in reps],
                       "how": "each repeat: barrier + sync, K steps event-timed on the launch stream, sync + "
                              "barrier; max over ranks per repeat; median over repeats"},
            "clocks": clocks,
            "cufft": cufft,
            "roundtrip_rel_l2": rt_err,
        }
        print(json.dumps(line), flush=True)
    ranks.close()
    return 0


def c2c_end_to_end(ranks, stream, x, tf):
    """Pinned host buffers through the public asynchronous call: H2D of every
    signal, forward, inverse, D2H, inside each step.  The batch moves in 16
    chunks over three streams so one chunk's upload, another's transforms and
    a third's download overlap (the copy directions use separate engines)."""
    import torch

    dev = ranks.dev
    hx = torch.empty(x.shape, dtype=x.dtype, pin_memory=True)
    hx.copy_(x)
    hz = torch.empty_like(hx, pin_memory=True)
    dx, dy, dz = torch.empty_like(x), torch.empty_like(x), torch.empty_like(x)
    e_steps = 3
    n_chunks = 16 if BATCH % 16 == 0 else 1
    csz = BATCH // n_chunks
    lanes = [torch.cuda.Stream(dev) for _ in range(3)]

    def e2e_step():
        start = torch.cuda.Event()
        start.record(stream)
        for s in lanes:
            s.wait_event(start)
        for c in range(n_chunks):
            s, sl = lanes[c % 3], slice(c * csz, (c + 1) * csz)
            with torch.cuda.stream(s):
                dx[sl].copy_(hx[sl], non_blocking=True)
            tf.c2c_async(DTYPE, N, True, dx[sl], dy[sl], csz, s)
            tf.c2c_async(DTYPE, N, False, dy[sl], dz[sl], csz, s)
            with torch.cuda.stream(s):
                hz[sl].copy_(dz[sl], non_blocking=True)
        for s in lanes:
            done = torch.cuda.Event()
            done.record(s)
            stream.wait_event(done)

    e2e_step()
    tf.sync_check(stream)
    torch.cuda.synchronize(dev)
    ranks.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e_steps):
        e2e_step()
    e1.record(stream)
    tf.sync_check(stream)
    torch.cuda.synchronize(dev)
    for s in lanes:
        tf.sync_check(s)
    if not torch.equal(hz[:4].to(dev), dz[:4]):
        raise RuntimeError("end-to-end result differs from the device result")
    ems = ranks.max(e0.elapsed_time(e1))
    return {"value": ranks.world * e_steps * 2 * BYTES_PER_TRANSFORM_BATCH / (ems / 1e3) / 1e9, "unit": "GB/s",
            "h2d_bytes_per_step": int(hx.numel() * hx.element_size()),
            "d2h_bytes_per_step": int(hz.numel() * hz.element_size()),
            "ms_per_step": ems / e_steps, "chunks": n_chunks, "streams": len(lanes)}


def run_conv2d(args):
    """Config 5 on 1..8 GPUs: each rank convolves its share of the images
    (strong: the 64 batch images split by image pair; weak: all of them) with
    one thff_conv2d call per step; no collective touches image data."""
    import torch
    import thunderfft_b200 as tf
    from thunderfft_b200.shard import conv2d_image_shard

    ranks = Ranks()
    world, rank, dev = ranks.world, ranks.rank, ranks.dev
    stream = torch.cuda.current_stream(dev)
    tf.conv2d_set_arithmetic(args.conv_arith)
    b0, nb = conv2d_image_shard(CONV2D_B, world, rank, args.scaling)
    C, hw, f = CONV2D_C, CONV2D_HW, CONV2D_F
    g = torch.Generator(device=dev)
    g.manual_seed(4321)   # the same filters on every rank
    filt = torch.randn(C, f, f, device=dev, generator=g)
    g.manual_seed(5000 + b0 if args.scaling == "strong" else 5000 + 97 * rank)
    x = torch.randn(nb, C, hw, hw, device=dev, generator=g)
    y = torch.empty_like(x)
    tf.ThunderFFTInitialize("float", hw)
    spec = tf.conv2d_filter_spectra(filt, hw, hw)
    pairs = ((nb + 1) // 2) * C
    ws = tf.conv2d_workspace(hw, hw, pairs)
    bytes_per_step = 2 * x.numel() * 4

    def step():
        tf.conv2d(x, spec, ws, out=y, stream=stream, sync=False)

    for _ in range(max(args.warmup, 3)):
        step()
    tf.sync_check(stream)
    # correctness gate on sampled images of this very run (FP64 direct)
    import oracle

    pick = [(0, 0), (nb - 1, C - 1)]
    xs = np.stack([x[b, c].double().cpu().numpy() for b, c in pick])
    ref = oracle.circconv2d(xs, filt.double().cpu().numpy(), np.array([c for _, c in pick], np.int32))
    got = np.stack([y[b, c].double().cpu().numpy() for b, c in pick])
    gate_err = oracle.rel_l2(got, ref)
    if not gate_err <= 5e-3:
        raise RuntimeError(f"conv2d rel-L2 {gate_err} fails the 5e-3 gate")

    ms_max, reps, launches, clocks = timed_region(ranks, stream, args.steps, step, tf)
    # whole-job bytes: strong = the config's images once per step; weak = every rank's
    job_images = CONV2D_B * C if args.scaling == "strong" else world * CONV2D_B * C
    value = args.steps * job_images * hw * hw * 8 / (ms_max / 1e3) / 1e9
    per_call_us = ms_max / args.steps * 1e3
    achieved = bytes_per_step / (per_call_us / 1e6) / 1e9

    e2e = None
    if not args.no_extras:
        try:
            e2e = conv2d_end_to_end(ranks, stream, x, spec, tf, job_images)
        except Exception as e:  # pragma: no cover
            e2e = {"error": str(e)}

    peak, peak_kind = measured_peaks()
    if rank == 0:
        cpu = None
        if not (args.no_cpu_baseline or world > 1):
            v, imgs, dt, thr = conv2d_cpu_sample()
            cpu = {"value": v, "unit": "GB/s", "cores": thr, "kind": "port",
                   "sample": f"{imgs} images of 512x512, 31x31 filter, FP64 direct circular convolution, "
                             f"{dt:.1f} s on {thr} threads"}
        line = {
            "metric": CONV2D_METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": max(args.warmup, 3), "ms_per_step": ms_max / args.steps, "higher_is_better": True,
            "scaling": args.scaling, "vs_baseline": None, "dtype": "f16" if args.conv_arith == "mixed" else "tf32",
            "data": "synthetic",
            "config": {"workload": f"conv2d (BASELINE config 5): {CONV2D_B}x{C} fp32 {hw}x{hw} images, {f}x{f} "
                                   f"filter per channel, circular; {args.scaling} scaling, {nb} batch images per "
                                   "rank (rank 0)",
                       "images_per_job": job_images, "arithmetic": args.conv_arith,
                       "parallelism": f"batch-shard by image pair x{world}, no collective",
                       "l2": f"{x.numel() * 4 >> 20} MiB of images per rank"
                             + (" > 126 MB L2" if x.numel() * 4 > 126e6 else " (WARNING: fits in L2)")},
            "images_per_s": args.steps * job_images / (ms_max / 1e3),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak,
                         "traffic": profile_value("conv2d_config5.md", "traffic_bytes_per_call"),
                         "kernel": "thff_conv2d call (all passes), algorithmic 8 B per pixel",
                         "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                         else "fallback 6650 GB/s"},
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": launches,
            "timing": {"repeats": len(reps), "steps_per_repeat": args.steps,
                       "ms_min": min(reps), "ms_median": ms_max, "ms_max": max(reps),
                       "ms_each": [round(v, 4) for v in reps]},
            "clocks": clocks,
            "gate_rel_l2": gate_err,
        }
        print(json.dumps(line), flush=True)
    ranks.close()
    return 0


def conv2d_end_to_end(ranks, stream, x, spec, tf, job_images):
    """Pinned host images through thff_conv2d: per step, upload every image,
    convolve, download every result.  The rank's images move in chunks of
    image pairs over three streams (one workspace each) so uploads,
    convolutions and downloads of different chunks overlap."""
    import torch

    dev = ranks.dev
    nb, C, hw, _ = x.shape
    hx = torch.empty(x.shape, dtype=x.dtype, pin_memory=True)
    hx.copy_(x)
    hy = torch.empty_like(hx, pin_memory=True)
    dx, dy = torch.empty_like(x), torch.empty_like(x)
    per = 2                                   # batch images per chunk (one pair per channel)
    chunks = [(b, min(per, nb - b)) for b in range(0, nb, per)]
    lanes = [torch.cuda.Stream(dev) for _ in range(3)]
    wss = [tf.conv2d_workspace(hw, hw, C) for _ in lanes]
    e_steps = 2

    def e2e_step():
        start = torch.cuda.Event()
        start.record(stream)
        for s in lanes:
            s.wait_event(start)
        for i, (b, k) in enumerate(chunks):
            s, ws = lanes[i % 3], wss[i % 3]
            with torch.cuda.stream(s):
                dx[b:b + k].copy_(hx[b:b + k], non_blocking=True)
            tf.conv2d(dx[b:b + k], spec, ws, out=dy[b:b + k], stream=s, sync=False)
            with torch.cuda.stream(s):
                hy[b:b + k].copy_(dy[b:b + k], non_blocking=True)
        for s in lanes:
            done = torch.cuda.Event()
            done.record(s)
            stream.wait_event(done)

    e2e_step()
    torch.cuda.synchronize(dev)
    for s in lanes:
        tf.sync_check(s)
    ranks.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    for s in lanes:
        tf.sync_check(s)
    if not torch.equal(hy[:1].to(dev), dy[:1]):
        raise RuntimeError("end-to-end result differs from the device result")
    ems = ranks.max(e0.elapsed_time(e1))
    return {"value": e_steps * job_images * hw * hw * 8 / (ems / 1e3) / 1e9, "unit": "GB/s",
            "h2d_bytes_per_step": int(hx.numel() * 4), "d2h_bytes_per_step": int(hy.numel() * 4),
            "ms_per_step": ems / e_steps, "chunks": len(chunks), "streams": len(lanes)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="c2c", choices=["c2c", "conv2d"],
                    help="c2c: BASELINE config 2 (the contract line); conv2d: config 5")
    ap.add_argument("--scaling", default="strong", choices=["strong", "weak"],
                    help="conv2d: strong = the config's 2048 images split across ranks; weak = all on every rank")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--n", type=int, default=1024, help="transform length (default: config 2)")
    ap.add_argument("--batch", type=int, default=65536, help="signals per GPU")
    ap.add_argument("--dtype", default="float", choices=["float", "half"])
    ap.add_argument("--no-extras", action="store_true", help="skip cuFFT, e2e and CPU legs (profiling)")
    ap.add_argument("--no-cufft", action="store_true", help="sweep: skip the cuFFT columns")
    ap.add_argument("--sweep", action="store_true",
                    help="print the per-size table (all N, both storage types, conv kernels) instead of the JSON line")
    ap.add_argument("--sweep-scale", type=int, default=1, help="divide the sweep's batches by this (profiling)")
    ap.add_argument("--no-conv", action="store_true", help="sweep: skip the conv1d / conv2d rows")
    ap.add_argument("--conv-arith", default="mixed", choices=["mixed", "tf32"],
                    help="arithmetic of the conv1d / conv2d rows (default: the library default, mixed)")
    ap.add_argument("--tiled-taps", type=int, default=9, help="sweep: filter taps of the tiled conv1d row (1..64)")
    ap.add_argument("--sweep-only", default="all", choices=["all", "fft", "conv1d", "conv2d", "tiled"],
                    help="sweep: run only these rows (profiling one kernel)")
    args = ap.parse_args()
    configure(args.n, args.batch, args.dtype)
    if args.no_extras:
        args.no_cpu_baseline = True
    if args.sweep:
        return run_sweep(args)
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == "conv2d":
        return run_conv2d(args)
    return run_c2c(args)


if __name__ == "__main__":
    sys.exit(main())
