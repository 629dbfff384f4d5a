"""C ABI checks that need no GPU: the library loads, exports every symbol the
public C header declares, and enforces the reference wrapper's argument
contract before any CUDA call (sample/validation/fft_validation.cu:331-352,
the 18 host-only checks, restated for the C ABI and the Python mirror)."""
import ctypes
import re
from pathlib import Path

import pytest

import thunderfft_b200 as tf

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols():
    syms = set()
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        for m in re.finditer(r"\b(thff_\w+)\s*\(", text):
            syms.add(m.group(1))
    return sorted(syms)


def test_library_loads_and_exports_declared_symbols():
    lib = tf.load_library()
    syms = declared_symbols()
    assert len(syms) >= 7
    for s in syms:
        assert hasattr(lib, s), f"missing export {s}"
    assert "sm_100a" in tf.version()


def test_library_is_in_tree():
    assert tf.library_path().resolve().parent == (ROOT / "thunderfft_b200").resolve()


@pytest.mark.parametrize("T", ["float", "half"])
def test_host_argument_contract_python(T):
    value = 0x1000  # a host pointer value that must never be dereferenced
    with pytest.raises(ValueError):
        tf.ThunderFFT_global(T, 64, True, 0, 0, -1)
    with pytest.raises(ValueError):
        tf.ThunderFFT_global(T, 64, True, 0, value, 1)
    with pytest.raises(ValueError):
        tf.ThunderFFT_global(T, 64, True, value, 0, 1)
    with pytest.raises(ValueError):
        tf.ThunderFFT_global(T, 64, True, value, value, 1)
    tf.ThunderFFT_global(T, 64, True, 0, 0, 0)  # zero batch: no-op
    for n in (-1, 0, 32, 8192):
        with pytest.raises(ValueError):
            tf.ThunderFFTInitialize(T, n)


@pytest.mark.parametrize("dtype", [0, 1])
def test_host_argument_contract_c_abi(dtype):
    lib = tf.load_library()
    v = ctypes.c_void_p(0x1000)
    null = ctypes.c_void_p(0)
    assert lib.thff_global(dtype, 64, 1, null, null, -1, null) == tf.THFF_INVALID_ARGUMENT
    assert lib.thff_global(dtype, 64, 1, null, v, 1, null) == tf.THFF_INVALID_ARGUMENT
    assert lib.thff_global(dtype, 64, 1, v, null, 1, null) == tf.THFF_INVALID_ARGUMENT
    assert lib.thff_global(dtype, 64, 1, v, v, 1, null) == tf.THFF_INVALID_ARGUMENT
    assert lib.thff_global(dtype, 64, 1, null, null, 0, null) == tf.THFF_OK
    # overlapping (not identical) buffers are rejected too
    assert lib.thff_global(dtype, 64, 1, v, ctypes.c_void_p(0x1000 + 64), 4, null) == tf.THFF_INVALID_ARGUMENT
    for n in (-1, 0, 32, 8192, 100):
        assert lib.thff_initialize(dtype, n) == tf.THFF_INVALID_ARGUMENT
        assert lib.thff_global(dtype, n, 1, v, ctypes.c_void_p(0x100000), 1, null) == tf.THFF_INVALID_ARGUMENT
    assert b"unsupported" in lib.thff_last_error().lower() or b"length" in lib.thff_last_error().lower()


def test_bad_dtype_rejected():
    lib = tf.load_library()
    assert lib.thff_initialize(7, 64) == tf.THFF_INVALID_ARGUMENT
    assert lib.thff_finalize(-1) == tf.THFF_INVALID_ARGUMENT
    with pytest.raises(ValueError):
        tf.ThunderFFTInitialize("double", 64)


def test_errors_map_to_exceptions():
    # status -> exception mapping of the Python mirror (invalid_argument vs runtime_error)
    with pytest.raises(ValueError):
        tf._check(tf.THFF_INVALID_ARGUMENT)
    for st in (tf.THFF_CUDA_ERROR, tf.THFF_DEVICE_TIMEOUT, tf.THFF_UNSUPPORTED):
        with pytest.raises(RuntimeError):
            tf._check(st)
