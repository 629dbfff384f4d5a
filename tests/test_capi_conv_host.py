"""Host-side argument contract of the convolution entry points of the C ABI
(include/thff.h), checked without a GPU.

Every check below is decided before the library touches CUDA, so a CPU-only
machine returns the same status codes as a B200.  The reference samples
(sample/conv1d/conv1d_fullfft_l4096_thunder.cu, sample/conv1d/main.cu,
sample/conv2d/thunder.cu) hard-code their shapes and have no argument
checks of their own; these follow the conventions of the reference wrapper
(sample/validation/fft_validation.cu:331-352): negative batch and bad sizes
are invalid arguments, a zero batch is a no-op before any CUDA call, null
and misaligned pointers are invalid arguments."""
import ctypes

import pytest

import thunderfft_b200 as tf

V = ctypes.c_void_p(0x100000)   # 16-byte aligned host value, never dereferenced
V2 = ctypes.c_void_p(0x200000)
V3 = ctypes.c_void_p(0x300000)
NULL = ctypes.c_void_p(0)
F32, F16 = 0, 1
INVALID, OK = tf.THFF_INVALID_ARGUMENT, tf.THFF_OK


@pytest.fixture(scope="module")
def lib():
    lib = tf.load_library()
    vp, i32, i64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong
    lib.thff_conv2d_noalloc.argtypes = [i32, i64, i32, i32, i32, vp, vp, vp, vp]
    lib.thff_conv2d_noalloc.restype = i32
    return lib


def last_error(lib):
    return lib.thff_last_error().decode()


def test_size_queries(lib):
    assert lib.thff_conv1d_spectrum_bytes(F32, 1024) == 1024 * 8
    assert lib.thff_conv1d_spectrum_bytes(F32, 4096) == 4096 * 8
    for dtype, n in ((F16, 1024), (F32, 2048), (F32, 0)):
        assert lib.thff_conv1d_spectrum_bytes(dtype, n) == -1
    assert lib.thff_conv1d_tiled_operator_bytes(F32) == 128 * 128 * 4
    assert lib.thff_conv1d_tiled_operator_bytes(F16) == 128 * 128 * 2
    assert lib.thff_conv1d_tiled_operator_bytes(5) == -1
    # one image pair = one complex 2-D transform of h*w float2 values
    assert lib.thff_conv2d_workspace_bytes(F32, 128, 256, 1) == 2 * 128 * 256 * 8
    assert lib.thff_conv2d_workspace_bytes(F32, 4096, 4096, 3) == 3 * 2 * 4096 * 4096 * 8
    for dtype, h, w, pairs in ((F16, 128, 128, 1), (F32, 192, 128, 1), (F32, 128, 8192, 1),
                               (F32, 128, 128, 0), (F32, 64, 128, 1)):
        assert lib.thff_conv2d_workspace_bytes(dtype, h, w, pairs) == -1


@pytest.mark.parametrize("fn", ["thff_conv1d_async", "thff_conv1d"])
def test_conv1d_contract(lib, fn):
    call = getattr(lib, fn)
    assert call(F32, 1024, 1024, V, V2, V3, 0, NULL) == OK          # zero batch: no-op
    assert call(F16, 1024, 1024, V, V2, V3, 1, NULL) == INVALID     # float storage only
    for n in (512, 2048, 8192):
        assert call(F32, n, 512, V, V2, V3, 1, NULL) == INVALID
    # lin: positive multiple of sqrt(n) (32 or 64), at most n
    for n, lin in ((1024, 0), (1024, 33), (1024, 1056), (4096, 32), (4096, 4160), (4096, -64)):
        assert call(F32, n, lin, V, V2, V3, 1, NULL) == INVALID, (n, lin)
        assert "input length" in last_error(lib)
    assert call(F32, 1024, 1024, V, V2, V3, -1, NULL) == INVALID
    for x, s, y in ((NULL, V2, V3), (V, NULL, V3), (V, V2, NULL)):
        assert call(F32, 1024, 1024, x, s, y, 1, NULL) == INVALID
    # x and the spectrum 16-byte aligned, y 8-byte aligned
    assert call(F32, 1024, 1024, ctypes.c_void_p(0x100008), V2, V3, 1, NULL) == INVALID
    assert call(F32, 1024, 1024, V, ctypes.c_void_p(0x200008), V3, 1, NULL) == INVALID
    assert call(F32, 1024, 1024, V, V2, ctypes.c_void_p(0x300004), 1, NULL) == INVALID
    assert "aligned" in last_error(lib)


def test_conv1d_filter_spectrum_contract(lib):
    call = lib.thff_conv1d_filter_spectrum
    assert call(F16, 1024, V, 8, V2, NULL) == INVALID
    assert call(F32, 2048, V, 8, V2, NULL) == INVALID
    for taps in (0, -3, 1025):
        assert call(F32, 1024, V, taps, V2, NULL) == INVALID
    assert call(F32, 4096, NULL, 8, V2, NULL) == INVALID
    assert call(F32, 4096, V, 8, NULL, NULL) == INVALID


@pytest.mark.parametrize("fn", ["thff_conv1d_tiled_async", "thff_conv1d_tiled"])
@pytest.mark.parametrize("dtype", [F32, F16])
def test_conv1d_tiled_contract(lib, fn, dtype):
    call = getattr(lib, fn)
    assert call(dtype, 1 << 20, 9, V, V2, V3, 0, NULL) == OK        # zero batch: no-op
    assert call(7, 1 << 20, 9, V, V2, V3, 1, NULL) == INVALID
    for f in (0, 65, -1):
        assert call(dtype, 1 << 20, f, V, V2, V3, 1, NULL) == INVALID
        assert "filter length" in last_error(lib)
    assert call(dtype, 8, 9, V, V2, V3, 1, NULL) == INVALID          # input shorter than the filter
    assert call(dtype, 9, 9, V, V2, V3, 0, NULL) == OK                # exactly one output is allowed
    assert call(dtype, 1 << 20, 9, V, V2, V3, -2, NULL) == INVALID
    for x, op, y in ((NULL, V2, V3), (V, NULL, V3), (V, V2, NULL)):
        assert call(dtype, 1 << 20, 9, x, op, y, 1, NULL) == INVALID
    # x and y aligned to one complex element (4 B half2, 8 B float2), operator to 16 B
    esz = 4 if dtype == F16 else 8
    assert call(dtype, 1 << 20, 9, ctypes.c_void_p(0x100000 + esz // 2), V2, V3, 1, NULL) == INVALID
    assert call(dtype, 1 << 20, 9, V, V2, ctypes.c_void_p(0x300000 + esz // 2), 1, NULL) == INVALID
    assert call(dtype, 1 << 20, 9, V, ctypes.c_void_p(0x200008), V3, 1, NULL) == INVALID


def test_conv1d_tiled_operator_contract(lib):
    call = lib.thff_conv1d_tiled_operator
    assert call(3, V, 9, V2, NULL) == INVALID
    for f in (0, 65):
        assert call(F32, V, f, V2, NULL) == INVALID
    assert call(F32, NULL, 9, V2, NULL) == INVALID
    assert call(F16, V, 9, NULL, NULL) == INVALID
    assert call(F32, V, 9, ctypes.c_void_p(0x200008), NULL) == INVALID   # operator 16-byte aligned
    assert call(F32, ctypes.c_void_p(0x100004), 9, V2, NULL) == INVALID  # filter 8-byte aligned


@pytest.mark.parametrize("fn", ["thff_conv2d_async", "thff_conv2d"])
def test_conv2d_contract(lib, fn):
    call = getattr(lib, fn)
    ws = 2 * 256 * 256 * 8
    V4 = ctypes.c_void_p(0x400000)
    assert call(F32, 0, 3, 256, 256, V, V2, V3, V4, ws, NULL) == OK    # zero batch: no-op
    assert call(F16, 2, 3, 256, 256, V, V2, V3, V4, ws, NULL) == INVALID
    for h, w in ((64, 256), (256, 8192), (192, 256), (256, 0)):
        assert call(F32, 2, 3, h, w, V, V2, V3, V4, ws, NULL) == INVALID
        assert "image sides" in last_error(lib)
    assert call(F32, -1, 3, 256, 256, V, V2, V3, V4, ws, NULL) == INVALID
    assert call(F32, 2, 0, 256, 256, V, V2, V3, V4, ws, NULL) == INVALID
    for ptrs in ((NULL, V2, V3, V4), (V, NULL, V3, V4), (V, V2, NULL, V4), (V, V2, V3, NULL)):
        assert call(F32, 2, 3, 256, 256, *ptrs, ws, NULL) == INVALID
    odd = ctypes.c_void_p(0x100008)
    for ptrs in ((odd, V2, V3, V4), (V, odd, V3, V4), (V, V2, odd, V4), (V, V2, V3, odd)):
        assert call(F32, 2, 3, 256, 256, *ptrs, ws, NULL) == INVALID
    assert call(F32, 2, 3, 256, 256, V, V2, V3, V4, ws - 16, NULL) == INVALID
    assert "workspace" in last_error(lib)


def test_conv2d_filter_spectra_contract(lib):
    call = lib.thff_conv2d_filter_spectra
    V4 = ctypes.c_void_p(0x400000)
    need = 3 * 5 * 256 * 16   # channels * f * w * 16 bytes
    assert call(F16, 256, 256, 3, 5, V, V2, V4, need, NULL) == INVALID
    assert call(F32, 100, 256, 3, 5, V, V2, V4, need, NULL) == INVALID
    for chans, f in ((0, 5), (3, 0), (3, 257)):
        assert call(F32, 256, 256, chans, f, V, V2, V4, need, NULL) == INVALID
    assert call(F32, 256, 256, 3, 5, NULL, V2, V4, need, NULL) == INVALID
    assert call(F32, 256, 256, 3, 5, V, NULL, V4, need, NULL) == INVALID
    assert call(F32, 256, 256, 3, 5, V, V2, NULL, need, NULL) == INVALID
    assert call(F32, 256, 256, 3, 5, V, V2, V4, need - 1, NULL) == INVALID
    assert "workspace" in last_error(lib)


def test_conv2d_noalloc_contract(lib):
    call = lib.thff_conv2d_noalloc
    assert call(F32, 0, 3, 1024, 1024, V, V2, V3, NULL) == OK         # largest pair that fits, zero batch
    # h*w above 1048576 does not fit the fixed scratch: rejected even for a zero batch
    for h, w in ((2048, 1024), (1024, 2048), (4096, 4096)):
        assert call(F32, 0, 3, h, w, V, V2, V3, NULL) == INVALID
        assert "1048576" in last_error(lib)
    assert call(F16, 2, 3, 256, 256, V, V2, V3, NULL) == INVALID
    assert call(F32, 2, 3, 96, 256, V, V2, V3, NULL) == INVALID
    assert call(F32, -2, 3, 256, 256, V, V2, V3, NULL) == INVALID
    assert call(F32, 2, -1, 256, 256, V, V2, V3, NULL) == INVALID
    for ptrs in ((NULL, V2, V3), (V, NULL, V3), (V, V2, NULL)):
        assert call(F32, 2, 3, 256, 256, *ptrs, NULL) == INVALID
    odd = ctypes.c_void_p(0x100004)
    for ptrs in ((odd, V2, V3), (V, odd, V3), (V, V2, odd)):
        assert call(F32, 2, 3, 256, 256, *ptrs, NULL) == INVALID


def test_set_arithmetic_contract(lib):
    for setter in (lib.thff_conv1d_set_arithmetic, lib.thff_conv2d_set_arithmetic):
        for bad in (-1, 2, 99):
            assert setter(bad) == INVALID
            assert "arithmetic" in last_error(lib)
        assert setter(1) == OK   # THFF_CONV_TF32
        assert setter(0) == OK   # THFF_CONV_MIXED, the default, restored
