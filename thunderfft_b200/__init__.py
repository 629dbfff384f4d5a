"""thunderfft_b200 — B200-native (sm_100a) tensor-core batched FFT.

Python mirror of the ThunderFFT host API over the C ABI of
``libthunderfft_b200.so`` (include/thff.h).  The names follow the reference's
header API (include/thunderfft/thunderfft.cuh):

=====================================  =======================================
reference (C++ templates)              here
=====================================  =======================================
``ThunderFFTInitialize<T>(N)``         ``ThunderFFTInitialize(T, N)``
``ThunderFFTFinalize<T>()``            ``ThunderFFTFinalize(T)``
``ThunderFFT_global<T,N,fwd>(i,o,b,s)`` ``ThunderFFT_global(T, N, fwd, i, o, b, s)``
=====================================  =======================================

``T`` is ``"float"`` (float2 storage, TF32 tensor-core arithmetic) or
``"half"`` (half2 storage, FP16 tensor-core arithmetic).  Argument errors raise
``ValueError`` (the reference's ``std::invalid_argument``); CUDA failures and
device-side timeouts raise ``RuntimeError`` (``std::runtime_error``).

There is no CPU fallback: every entry point needs the compiled library and a
B200; a missing ``.so`` raises at first use.

Convenience wrappers on torch tensors (``fft``, ``ifft``) are provided for
tests and benchmarks; torch is only used for device memory and streams.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path
from typing import Optional

__all__ = [
    "ThunderFFTInitialize", "ThunderFFTFinalize", "ThunderFFT_global", "c2c_async", "sync_check",
    "twiddle_table", "fft", "load_library", "library_path", "SUPPORTED_N", "batch_per_block",
    "warp_per_block", "threads_per_warp", "version", "conv1d_filter_spectrum", "conv1d",
    "conv2d_filter_spectra", "conv2d", "conv2d_workspace", "conv1d_set_arithmetic", "conv2d_set_arithmetic",
    "conv1d_tiled_operator", "conv1d_tiled", "launch_count",
]

SUPPORTED_N = (64, 128, 256, 512, 1024, 2048, 4096)
# Launch tuples of the reference header (detail/thunderfft_impl.cuh:14-32);
# kept for API compatibility of the device-side composition helpers.
batch_per_block = {64: 16, 128: 8, 256: 16, 512: 2, 1024: 1, 2048: 1, 4096: 1}
warp_per_block = {64: 1, 128: 1, 256: 4, 512: 1, 1024: 1, 2048: 2, 4096: 4}
threads_per_warp = 32

THFF_OK, THFF_INVALID_ARGUMENT, THFF_CUDA_ERROR, THFF_DEVICE_TIMEOUT, THFF_UNSUPPORTED = range(5)
_DTYPES = {"float": 0, "half": 1, "f32": 0, "f16": 1, "tf32": 0, "fp16": 1}

_PKG = Path(__file__).resolve().parent
_lib: Optional[ctypes.CDLL] = None


def library_path() -> Path:
    return Path(os.environ.get("THFF_LIBRARY", _PKG / "libthunderfft_b200.so"))


def load_library() -> ctypes.CDLL:
    """Load the compiled backend; raise if it is missing (no fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    path = library_path()
    if not path.exists():
        raise RuntimeError(
            f"[ThunderFFT] {path} is missing: build it with `python -m thunderfft_b200.build` "
            "(there is no CPU fallback)")
    lib = ctypes.CDLL(str(path))
    vp, i32, i64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong
    lib.thff_version.restype = ctypes.c_char_p
    lib.thff_last_error.restype = ctypes.c_char_p
    lib.thff_launch_count.argtypes = []
    lib.thff_launch_count.restype = ctypes.c_ulonglong
    lib.thff_initialize.argtypes = [i32, i32]
    lib.thff_finalize.argtypes = [i32]
    lib.thff_twiddle_table.argtypes = [i32, ctypes.POINTER(vp), ctypes.POINTER(i32)]
    lib.thff_global.argtypes = [i32, i32, i32, vp, vp, i32, vp]
    lib.thff_c2c_async.argtypes = [i32, i32, i32, vp, vp, i64, vp]
    lib.thff_sync_check.argtypes = [vp]
    lib.thff_conv1d_spectrum_bytes.argtypes = [i32, i32]
    lib.thff_conv1d_spectrum_bytes.restype = i64
    lib.thff_conv1d_filter_spectrum.argtypes = [i32, i32, vp, i32, vp, vp]
    lib.thff_conv1d_async.argtypes = [i32, i32, i32, vp, vp, vp, i64, vp]
    lib.thff_conv1d.argtypes = [i32, i32, i32, vp, vp, vp, i64, vp]
    lib.thff_conv2d_workspace_bytes.argtypes = [i32, i32, i32, i64]
    lib.thff_conv2d_workspace_bytes.restype = i64
    lib.thff_conv2d_filter_spectra.argtypes = [i32, i32, i32, i32, i32, vp, vp, vp, i64, vp]
    lib.thff_conv2d_filter_spectra.restype = i32
    lib.thff_conv2d_async.argtypes = [i32, i64, i32, i32, i32, vp, vp, vp, vp, i64, vp]
    lib.thff_conv2d_async.restype = i32
    lib.thff_conv2d.argtypes = [i32, i64, i32, i32, i32, vp, vp, vp, vp, i64, vp]
    lib.thff_conv2d.restype = i32
    lib.thff_selftest_wait_timeout.argtypes = [i32, vp]
    lib.thff_selftest_wait_timeout.restype = i32
    lib.thff_test_inject_cuda_error.argtypes = [i32, i32]
    lib.thff_test_inject_cuda_error.restype = i32
    lib.thff_conv1d_set_arithmetic.argtypes = [i32]
    lib.thff_conv1d_set_arithmetic.restype = i32
    lib.thff_conv2d_set_arithmetic.argtypes = [i32]
    lib.thff_conv2d_set_arithmetic.restype = i32
    lib.thff_conv1d_tiled_operator_bytes.argtypes = [i32]
    lib.thff_conv1d_tiled_operator_bytes.restype = i64
    lib.thff_conv1d_tiled_operator.argtypes = [i32, vp, i32, vp, vp]
    lib.thff_conv1d_tiled_operator.restype = i32
    lib.thff_conv1d_tiled_async.argtypes = [i32, i64, i32, vp, vp, vp, i64, vp]
    lib.thff_conv1d_tiled_async.restype = i32
    lib.thff_conv1d_tiled.argtypes = [i32, i64, i32, vp, vp, vp, i64, vp]
    lib.thff_conv1d_tiled.restype = i32
    for name in ("thff_initialize", "thff_finalize", "thff_twiddle_table", "thff_global",
                 "thff_c2c_async", "thff_sync_check", "thff_conv1d_filter_spectrum", "thff_conv1d_async",
                 "thff_conv1d"):
        getattr(lib, name).restype = i32
    _lib = lib
    return lib


def _dtype_code(T) -> int:
    key = T if isinstance(T, str) else getattr(T, "__name__", str(T))
    try:
        return _DTYPES[key]
    except KeyError:
        raise ValueError(f"ThunderFFT supports float and half only (got {T!r})") from None


def _check(status: int) -> None:
    if status == THFF_OK:
        return
    msg = load_library().thff_last_error().decode(errors="replace")
    if status == THFF_INVALID_ARGUMENT:
        raise ValueError(msg)
    raise RuntimeError(msg)


def version() -> str:
    return load_library().thff_version().decode()


def ThunderFFTInitialize(T, N: int) -> None:
    """Prepare twiddles/constants for length N on the current device
    (reference: ThunderFFTInitialize<T>(N), thunderfft_impl_twiddle.cuh:279-327)."""
    code = _dtype_code(T)
    if N not in SUPPORTED_N:  # before any CUDA call, like the reference
        raise ValueError("ThunderFFTInitialize<T>: unsupported FFT size")
    _check(load_library().thff_initialize(code, int(N)))


def ThunderFFTFinalize(T) -> None:
    """Release the current device's cached table (reference: ThunderFFTFinalize<T>())."""
    _check(load_library().thff_finalize(_dtype_code(T)))


def twiddle_table(T):
    """(device pointer, N) of the current device's cached twiddle table."""
    p, n = ctypes.c_void_p(), ctypes.c_int()
    _check(load_library().thff_twiddle_table(_dtype_code(T), ctypes.byref(p), ctypes.byref(n)))
    return (p.value or 0), n.value


def _ptr(x) -> int:
    if x is None:
        return 0
    if isinstance(x, int):
        return x
    return int(x.data_ptr())


def _stream_handle(stream) -> int:
    if stream is None:
        return 0
    if isinstance(stream, int):
        return stream
    return int(stream.cuda_stream)


def ThunderFFT_global(T, N: int, forward: bool, d_input, d_output, batch: int, stream=None) -> None:
    """Batched C2C FFT with the reference wrapper's contract
    (ThunderFFT_global<T,N,forward>, thunderfft_impl_kernel.cuh:6-41):
    batch < 0 -> ValueError; batch == 0 -> no-op before any CUDA or pointer
    access; null/identical pointers -> ValueError; synchronizes ``stream``.
    ``d_input``/``d_output`` are device pointers (int) or CUDA tensors."""
    code = _dtype_code(T)
    if N not in SUPPORTED_N:
        raise ValueError("Unsupported ThunderFFT length")
    if batch < 0:
        raise ValueError("ThunderFFT batch must be nonnegative")
    if batch == 0:
        return
    _check(load_library().thff_global(code, int(N), 1 if forward else 0, _ptr(d_input), _ptr(d_output),
                                      int(batch), _stream_handle(stream)))


def c2c_async(T, N: int, forward: bool, d_input, d_output, batch: int, stream=None) -> None:
    """Asynchronous form (64-bit batch; no stream synchronization)."""
    _check(load_library().thff_c2c_async(_dtype_code(T), int(N), 1 if forward else 0, _ptr(d_input),
                                         _ptr(d_output), int(batch), _stream_handle(stream)))


def launch_count() -> int:
    """Kernels the library has launched in this process (thff_launch_count)."""
    return int(load_library().thff_launch_count())


def sync_check(stream=None) -> None:
    """Synchronize ``stream`` and raise if a kernel recorded a device-side timeout."""
    _check(load_library().thff_sync_check(_stream_handle(stream)))


def fft(x, forward: bool = True, out=None, stream=None, sync: bool = True):
    """Transform the last axis of a CUDA tensor.

    ``x``: complex64 (float path) or float16 with a trailing axis of 2
    (re, im) (half path); last complex length in SUPPORTED_N; contiguous.
    Returns ``out`` (allocated like ``x`` when None)."""
    import torch

    if not x.is_cuda:
        raise ValueError("ThunderFFT operates on CUDA tensors only")
    if x.dtype == torch.complex64:
        T, n = "float", x.shape[-1]
    elif x.dtype == torch.float16 and x.shape[-1] == 2:
        T, n = "half", x.shape[-2]
    else:
        raise ValueError("expected complex64, or float16 with a trailing (re, im) axis")
    if not x.is_contiguous():
        raise ValueError("input must be contiguous")
    batch = x.numel() // (n if T == "float" else 2 * n)
    if out is None:
        out = torch.empty_like(x)
    c2c_async(T, n, forward, x, out, batch, stream if stream is not None else torch.cuda.current_stream())
    if sync:
        sync_check(stream if stream is not None else torch.cuda.current_stream())
    return out


def conv1d_filter_spectrum(h, n: int, stream=None):
    """Filter spectrum for `conv1d`: H[k] = (1/n) sum_j h[j] exp(-2 pi i j k / n)
    for a real float32 CUDA tensor h (taps <= n); returns a complex64 tensor."""
    import torch

    if not (h.is_cuda and h.dtype == torch.float32 and h.dim() == 1 and h.is_contiguous()):
        raise ValueError("filter must be a contiguous 1-D float32 CUDA tensor")
    spec = torch.empty(n, dtype=torch.complex64, device=h.device)
    st = stream if stream is not None else torch.cuda.current_stream(h.device)
    _check(load_library().thff_conv1d_filter_spectrum(0, int(n), h.data_ptr(), int(h.numel()), spec.data_ptr(),
                                                      _stream_handle(st)))
    return spec


def conv1d(x, spectrum, n: int, out=None, stream=None, sync: bool = True):
    """Fused real circular convolution of every row of x (float32 CUDA tensor
    [batch, lin], zero-padded to n) with the filter whose spectrum is given:
    out[b, m] = sum_k x[b][(m-k) mod n] h[k] (one kernel: FFT, multiply,
    inverse FFT).  Returns out [batch, n] float32."""
    import torch

    if not (x.is_cuda and x.dtype == torch.float32 and x.dim() == 2 and x.is_contiguous()):
        raise ValueError("x must be a contiguous [batch, lin] float32 CUDA tensor")
    batch, lin = x.shape
    if out is None:
        out = torch.empty(batch, n, dtype=torch.float32, device=x.device)
    st = stream if stream is not None else torch.cuda.current_stream(x.device)
    fn = load_library().thff_conv1d if sync else load_library().thff_conv1d_async
    _check(fn(0, int(n), int(lin), x.data_ptr(), spectrum.data_ptr(), out.data_ptr(), int(batch),
              _stream_handle(st)))
    return out


CONV_MIXED, CONV_TF32 = 0, 1


def conv1d_tiled_operator(filt, T="float", stream=None):
    """Operator of the tiled (overlap-save) convolution for the complex filter
    taps `filt` (complex64 CUDA tensor, 1 <= len <= 64), for storage type T
    (reference: the padded filter's cuFFT spectrum, sample/conv1d/main.cu:145-153)."""
    import torch

    if not (filt.is_cuda and filt.dtype == torch.complex64 and filt.dim() == 1 and filt.is_contiguous()):
        raise ValueError("filter must be a contiguous 1-D complex64 CUDA tensor")
    code = _dtype_code(T)
    lib = load_library()
    op = torch.empty(int(lib.thff_conv1d_tiled_operator_bytes(code)), dtype=torch.uint8, device=filt.device)
    st = stream if stream is not None else torch.cuda.current_stream(filt.device)
    _check(lib.thff_conv1d_tiled_operator(code, filt.data_ptr(), int(filt.numel()), op.data_ptr(),
                                          _stream_handle(st)))
    op.filter_length = int(filt.numel())
    return op


def conv1d_tiled(x, operator, f: Optional[int] = None, out=None, stream=None, sync: bool = True):
    """Tiled 64-point FFT convolution of every row of x (valid correlation
    with the operator's filter): x complex64 [batch, L] (float2 / TF32) or
    float16 [batch, L, 2] (half2 / FP16); returns [batch, L - f + 1] of the
    same type (reference: sample/conv1d/main.cu:38-129)."""
    import torch

    f = int(f if f is not None else getattr(operator, "filter_length"))
    if x.dtype == torch.complex64:
        T, L, shape = "float", x.shape[-1], lambda b, n: (b, n)
    elif x.dtype == torch.float16 and x.shape[-1] == 2:
        T, L, shape = "half", x.shape[-2], lambda b, n: (b, n, 2)
    else:
        raise ValueError("x must be complex64 [batch, L] or float16 [batch, L, 2]")
    if not (x.is_cuda and x.is_contiguous()):
        raise ValueError("x must be a contiguous CUDA tensor")
    batch = x.numel() // (L * (1 if T == "float" else 2))
    if out is None:
        out = torch.empty(shape(batch, L - f + 1), dtype=x.dtype, device=x.device)
    st = stream if stream is not None else torch.cuda.current_stream(x.device)
    fn = load_library().thff_conv1d_tiled if sync else load_library().thff_conv1d_tiled_async
    _check(fn(_dtype_code(T), int(L), f, x.data_ptr(), operator.data_ptr(), out.data_ptr(), int(batch),
              _stream_handle(st)))
    return out


def conv1d_set_arithmetic(mode) -> None:
    """Tensor-core arithmetic of the conv1d kernels (process-wide):
    "mixed" (default: TF32 first stage, FP16 operands with exact power-of-two
    range scaling for stages 2-4, FP32 accumulation) or "tf32"."""
    code = {"mixed": CONV_MIXED, "tf32": CONV_TF32}.get(mode, mode)
    _check(load_library().thff_conv1d_set_arithmetic(int(code)))


def conv2d_set_arithmetic(mode) -> None:
    """Arithmetic of conv2d (process-wide): "mixed" (default: half2
    intermediates with exact power-of-two range scaling, TF32 row pass on the
    fp32 images, FP16 passes with FP32 accumulation) or "tf32" (float2
    intermediates)."""
    code = {"mixed": CONV_MIXED, "tf32": CONV_TF32}.get(mode, mode)
    _check(load_library().thff_conv2d_set_arithmetic(int(code)))


def conv2d_workspace(h: int, w: int, pairs: int, device=None):
    """Allocate a conv2d workspace (uint8 CUDA tensor) for `pairs` image pairs per pass."""
    import torch

    n = load_library().thff_conv2d_workspace_bytes(0, int(h), int(w), int(pairs))
    if n <= 0:
        raise ValueError("unsupported conv2d shape")
    return torch.empty(n, dtype=torch.uint8, device=device or "cuda")


def conv2d_filter_spectra(filters, h: int, w: int, stream=None):
    """Spectra of real per-channel filters (float32 CUDA tensor [C, f, f]) for
    `conv2d`: complex64 [C, w, h] (transposed), 1/(h w) folded in."""
    import torch

    if not (filters.is_cuda and filters.dtype == torch.float32 and filters.dim() == 3 and filters.is_contiguous()):
        raise ValueError("filters must be a contiguous [C, f, f] float32 CUDA tensor")
    C, f, f2 = filters.shape
    if f != f2:
        raise ValueError("filters must be square")
    spec = torch.empty(C, w, h, dtype=torch.complex64, device=filters.device)
    ws = torch.empty(C * f * w * 16, dtype=torch.uint8, device=filters.device)
    st = stream if stream is not None else torch.cuda.current_stream(filters.device)
    _check(load_library().thff_conv2d_filter_spectra(0, int(h), int(w), int(C), int(f), filters.data_ptr(),
                                                      spec.data_ptr(), ws.data_ptr(), ws.numel(), _stream_handle(st)))
    return spec


def conv2d(x, spectra, workspace, out=None, stream=None, sync: bool = True):
    """Circular 2-D convolution of real images x (float32 CUDA [B, C, h, w])
    with per-channel filters given by `conv2d_filter_spectra`.  `workspace`
    is caller-owned scratch from `conv2d_workspace`."""
    import torch

    if not (x.is_cuda and x.dtype == torch.float32 and x.dim() == 4 and x.is_contiguous()):
        raise ValueError("x must be a contiguous [B, C, h, w] float32 CUDA tensor")
    B, C, h, w = x.shape
    if out is None:
        out = torch.empty_like(x)
    st = stream if stream is not None else torch.cuda.current_stream(x.device)
    fn = load_library().thff_conv2d if sync else load_library().thff_conv2d_async
    _check(fn(0, int(B), int(C), int(h), int(w), x.data_ptr(), spectra.data_ptr(), out.data_ptr(),
              workspace.data_ptr(), workspace.numel(), _stream_handle(st)))
    return out
