"""TEST INFRASTRUCTURE ONLY — FP64 CPU oracle for the ThunderFFT hot path.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg may use
this package, and only as the checker (or the timed CPU baseline); the
library's product path never imports it.

The oracle is ``thff_oracle.cpp`` (C++, compiled to ``oracle/_build``): FP64
radix-2 FFT / naive DFT, direct circular convolutions, and bit-exact copies of
the reference validation's seeded input generators.  See that file's header
for the reference lines each function follows and how parity is pinned.
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
SRC = HERE / "thff_oracle.cpp"
LIB = HERE / "_build" / "libthff_oracle.so"

_lib = None


def build(force: bool = False) -> Path:
    if not force and LIB.exists() and LIB.stat().st_mtime >= SRC.stat().st_mtime:
        return LIB
    LIB.parent.mkdir(parents=True, exist_ok=True)
    tmp = LIB.with_suffix(".tmp.so")
    subprocess.run(["g++", "-O2", "-std=c++17", "-shared", "-fPIC", "-pthread", "-o", str(tmp), str(SRC)],
                   check=True)
    tmp.replace(LIB)
    return LIB


def lib():
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        L = ctypes.CDLL(str(LIB))
        dp, fp, i64, i32 = (ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_float),
                            ctypes.c_int64, ctypes.c_int)
        L.thff_oracle_fft_f64.argtypes = [dp, dp, i64, i64, i32, i32]
        L.thff_oracle_fft_f32io.argtypes = [fp, fp, i64, i64, i32, i32]
        L.thff_oracle_dft_f64.argtypes = [dp, dp, i64, i64, i32, i32]
        L.thff_oracle_circconv1d_f64.argtypes = [dp, dp, dp, i64, i64, i64, i32]
        L.thff_oracle_circconv2d_f64.argtypes = [dp, dp, ctypes.POINTER(ctypes.c_int32), dp, i64, i64, i64,
                                                 i64, i32]
        L.thff_oracle_make_validation_input.argtypes = [i32, i32, i32, fp]
        L.thff_oracle_make_fft1d_input.argtypes = [i32, fp]
        L.thff_oracle_make_paper_input.argtypes = [i32, i64, fp]
        L.thff_oracle_hardware_threads.restype = i32
        for name in ("thff_oracle_fft_f64", "thff_oracle_fft_f32io", "thff_oracle_dft_f64",
                     "thff_oracle_circconv1d_f64", "thff_oracle_circconv2d_f64"):
            getattr(L, name).restype = i32
        _lib = L
    return _lib


def _dp(a):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_double))


def _fp(a):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def hardware_threads() -> int:
    return lib().thff_oracle_hardware_threads()


def fft(x: np.ndarray, forward: bool = True, threads: int = 0) -> np.ndarray:
    """FP64 FFT along the last axis of a complex array (unnormalized inverse)."""
    x = np.ascontiguousarray(x, dtype=np.complex128)
    n = x.shape[-1]
    out = np.empty_like(x)
    rc = lib().thff_oracle_fft_f64(_dp(x.view(np.float64)), _dp(out.view(np.float64)), n, x.size // n,
                                   1 if forward else 0, threads)
    if rc != 0:
        raise ValueError("oracle fft: length must be a power of two")
    return out


def fft_f32io(x: np.ndarray, forward: bool = True, threads: int = 0) -> np.ndarray:
    """Same FFT on complex64 storage (FP64 arithmetic inside)."""
    x = np.ascontiguousarray(x, dtype=np.complex64)
    n = x.shape[-1]
    out = np.empty_like(x)
    rc = lib().thff_oracle_fft_f32io(_fp(x.view(np.float32)), _fp(out.view(np.float32)), n, x.size // n,
                                     1 if forward else 0, threads)
    if rc != 0:
        raise ValueError("oracle fft: length must be a power of two")
    return out


def dft(x: np.ndarray, forward: bool = True, threads: int = 0) -> np.ndarray:
    """Naive FP64 DFT (definition) along the last axis."""
    x = np.ascontiguousarray(x, dtype=np.complex128)
    n = x.shape[-1]
    out = np.empty_like(x)
    lib().thff_oracle_dft_f64(_dp(x.view(np.float64)), _dp(out.view(np.float64)), n, x.size // n,
                              1 if forward else 0, threads)
    return out


def circconv1d(x: np.ndarray, h: np.ndarray, threads: int = 0) -> np.ndarray:
    """y[b][m] = sum_k x[b][(m-k) mod n] h[k] (real, FP64)."""
    x = np.ascontiguousarray(x, dtype=np.float64)
    h = np.ascontiguousarray(h, dtype=np.float64)
    n = x.shape[-1]
    y = np.empty_like(x)
    rc = lib().thff_oracle_circconv1d_f64(_dp(x), _dp(h), _dp(y), n, h.size, x.size // n, threads)
    if rc != 0:
        raise ValueError("oracle circconv1d: bad arguments")
    return y


def corr1d_valid(x: np.ndarray, g: np.ndarray) -> np.ndarray:
    """Valid complex correlation y[b][i] = sum_{k<f} x[b][i + k] g[k],
    i < L - f + 1, in FP64 — the check of the reference's tiled conv1d sample
    (sample/conv1d/main.cu:157-172, reference_conv1d_valid)."""
    x = np.atleast_2d(np.asarray(x, dtype=np.complex128))
    g = np.asarray(g, dtype=np.complex128)
    # numpy.correlate(a, v)[k] = sum_n a[n + k] conj(v[n])
    return np.stack([np.correlate(row, np.conj(g), mode="valid") for row in x])


def circconv2d(x: np.ndarray, filters: np.ndarray, filt_index: np.ndarray, threads: int = 0) -> np.ndarray:
    """y[b] = x[b] (*) filters[filt_index[b]] (2-D circular, FP64)."""
    x = np.ascontiguousarray(x, dtype=np.float64)
    f = np.ascontiguousarray(filters, dtype=np.float64)
    idx = np.ascontiguousarray(filt_index, dtype=np.int32)
    B, H, W = x.shape
    F = f.shape[-1]
    y = np.empty_like(x)
    rc = lib().thff_oracle_circconv2d_f64(_dp(x), _dp(f), idx.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                                          _dp(y), H, W, F, B, threads)
    if rc != 0:
        raise ValueError("oracle circconv2d: bad arguments")
    return y


def make_validation_input(n: int, batch: int, kind: int) -> np.ndarray:
    """Reference validation inputs (fft_validation.cu:130-163), complex64."""
    out = np.empty(2 * n * batch, dtype=np.float32)
    lib().thff_oracle_make_validation_input(n, batch, kind, _fp(out))
    return out.view(np.complex64).reshape(batch, n)


def make_fft1d_input(batch: int) -> np.ndarray:
    out = np.empty(2 * 64 * batch, dtype=np.float32)
    lib().thff_oracle_make_fft1d_input(batch, _fp(out))
    return out.view(np.complex64).reshape(batch, 64)


def make_paper_input(n: int, batch: int) -> np.ndarray:
    out = np.empty(2 * n * batch, dtype=np.float32)
    lib().thff_oracle_make_paper_input(n, n * batch, _fp(out))
    return out.view(np.complex64).reshape(batch, n)


def rel_l2(got: np.ndarray, ref: np.ndarray) -> float:
    got = np.asarray(got, dtype=np.complex128)
    ref = np.asarray(ref, dtype=np.complex128)
    den = np.sqrt(np.sum(np.abs(ref) ** 2))
    num = np.sqrt(np.sum(np.abs(got - ref) ** 2))
    return float(num / den) if den > 0 else float(num)


def rel_linf(got: np.ndarray, ref: np.ndarray) -> float:
    got = np.asarray(got, dtype=np.complex128)
    ref = np.asarray(ref, dtype=np.complex128)
    m = np.max(np.abs(ref))
    e = np.max(np.abs(got - ref))
    return float(e / m) if m > 0 else float(e)


# ---------------------------------------------------------------------------
# The reference's own GPU implementation (oracle/_ref/libthff_ref.so, built by
# oracle/build_ref.py from the reference headers).  TEST INFRASTRUCTURE: used
# only to compare outputs and to time the reference beside this library.
# ---------------------------------------------------------------------------
REF_LIB = HERE / "_ref" / "libthff_ref.so"
_ref = None


def ref_available() -> bool:
    return REF_LIB.exists()


def ref_sample(name: str) -> Path:
    """Path of a reference sample binary built by oracle/build_ref.py
    (ref_conv1d_tiled, ref_conv1d_full, ref_paper_fft); may not exist."""
    return HERE / "_ref" / name


def ref_lib():
    global _ref
    if _ref is None:
        L = ctypes.CDLL(str(REF_LIB))
        vp, i32 = ctypes.c_void_p, ctypes.c_int
        L.thff_ref_initialize.argtypes = [i32, i32]
        L.thff_ref_finalize.argtypes = [i32]
        L.thff_ref_global.argtypes = [i32, i32, i32, vp, vp, i32, vp]
        L.thff_ref_last_error.restype = ctypes.c_char_p
        for n in ("thff_ref_initialize", "thff_ref_finalize", "thff_ref_global"):
            getattr(L, n).restype = i32
        _ref = L
    return _ref


def ref_global(dtype: str, n: int, forward: bool, d_in: int, d_out: int, batch: int, stream: int = 0) -> None:
    """Run the reference's ThunderFFT_global<T,N,forward> (synchronizes)."""
    L = ref_lib()
    code = 0 if dtype == "float" else 1
    if L.thff_ref_initialize(code, n) != 0:
        raise RuntimeError(L.thff_ref_last_error().decode())
    if L.thff_ref_global(code, n, 1 if forward else 0, d_in, d_out, batch, stream) != 0:
        raise RuntimeError(L.thff_ref_last_error().decode())
