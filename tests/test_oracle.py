"""Pin the FP64 oracle (test infrastructure) before trusting it as the checker.

* against numpy.fft (pocketfft, an independent FP64 implementation);
* against the analytic answers of the reference validation's own inputs
  (sample/validation/fft_validation.cu:130-163): an offset impulse is a pure
  phase ramp, a bin-aligned tone is a single bin, a constant is N*c in bin 0;
* against the committed golden fixtures (tests/golden/make_golden.py);
* the seeded validation inputs bit for bit against the reference's own
  generator (digests in tests/golden/ref_inputs.json);
* against the reference's own output: its ThunderFFT_global, recompiled for
  sm_100a and run on a B200, frozen in tests/golden/ref_gpu_outputs.npz
  (tests/golden/make_ref_gpu_golden.py).
"""
import hashlib
import json
from pathlib import Path

import numpy as np
import pytest

import oracle

SIZES = (64, 128, 256, 512, 1024, 2048, 4096)
GOLD = np.load(__import__("pathlib").Path(__file__).parent / "golden" / "golden_fft.npz")


@pytest.mark.parametrize("n", SIZES)
@pytest.mark.parametrize("forward", [True, False])
def test_fft_matches_numpy(n, forward):
    rng = np.random.default_rng(n)
    x = rng.standard_normal((5, n)) + 1j * rng.standard_normal((5, n))
    ref = np.fft.fft(x, axis=-1) if forward else np.fft.ifft(x, axis=-1) * n
    assert oracle.rel_l2(oracle.fft(x, forward), ref) < 1e-13


@pytest.mark.parametrize("n", (64, 256, 1024))
def test_dft_definition_matches_fft(n):
    rng = np.random.default_rng(1)
    x = rng.standard_normal((2, n)) + 1j * rng.standard_normal((2, n))
    for fwd in (True, False):
        assert oracle.rel_l2(oracle.dft(x, fwd), oracle.fft(x, fwd)) < 1e-12


@pytest.mark.parametrize("n", SIZES)
def test_reference_inputs_known_answers(n):
    batch = 6
    k = np.arange(n)
    # offset impulse (.75,.25) at (13b+7)%n -> X[k] = c * exp(-2 pi i k m / n)
    x = oracle.make_validation_input(n, batch, 1)
    X = oracle.fft(x)
    for b in range(batch):
        m = (13 * b + 7) % n
        assert x[b, m] == np.complex64(0.75 + 0.25j) and np.count_nonzero(x[b]) == 1
        expect = (0.75 + 0.25j) * np.exp(-2j * np.pi * k * m / n)
        assert np.max(np.abs(X[b] - expect)) < 1e-12
    # tone f = 1 + (7b) % (n-1): single bin of magnitude n * 0.5 at k = f
    x = oracle.make_validation_input(n, batch, 2)
    X = oracle.fft(x)
    for b in range(batch):
        f = 1 + (7 * b) % (n - 1)
        assert abs(abs(X[b, f]) - 0.5 * n) < 1e-3 * n
        rest = np.delete(np.abs(X[b]), f)
        assert rest.max() < 1e-4 * n
    # constant (.25, -.125): bin 0 = n * c, other bins ~0
    x = oracle.make_validation_input(n, batch, 3)
    X = oracle.fft(x)
    assert np.allclose(X[:, 0], n * (0.25 - 0.125j), rtol=0, atol=1e-9)
    assert np.abs(X[:, 1:]).max() < 1e-9
    # gaussian: RMS 1 per signal
    x = oracle.make_validation_input(n, batch, 0)
    rms = np.sqrt(np.mean(np.abs(x.astype(np.complex128)) ** 2, axis=1))
    assert np.allclose(rms, 1.0, atol=1e-5)


def test_golden_fixtures_reproduced():
    for key in GOLD.files:
        if key.endswith("_fwd") and key.replace("_fwd", "_x") in GOLD.files:
            x = GOLD[key.replace("_fwd", "_x")]
            assert oracle.rel_l2(oracle.fft(x, True), GOLD[key]) < 1e-13, key
    assert oracle.rel_l2(oracle.fft(GOLD["cfg1_x"], False), GOLD["cfg1_inv"]) < 1e-13
    # the committed fixtures' inputs are the oracle's current generator output
    for n in (64, 256, 1024):
        for kind in range(4):
            assert np.array_equal(oracle.make_validation_input(n, 2, kind), GOLD[f"val_n{n}_k{kind}_x"])
    assert np.array_equal(oracle.make_fft1d_input(16), GOLD["fft1d_x"])


REF_INPUTS = json.loads((Path(__file__).parent / "golden" / "ref_inputs.json").read_text())


@pytest.mark.parametrize("n", SIZES)
@pytest.mark.parametrize("kind", range(4))
def test_validation_inputs_bit_equal_to_reference(n, kind):
    """The oracle's restatement of the reference validation's make_input
    (sample/validation/fft_validation.cu:130-163) reproduces the reference's
    compiled generator bit for bit at the program's default batch: the
    SHA-256 digests in tests/golden/ref_inputs.json come from the reference's
    own make_input (tests/golden/make_ref_inputs.py).  Kind 0 depends on
    g++ evaluating make_float2(normal(random), normal(random)) right to left."""
    x = oracle.make_validation_input(n, REF_INPUTS["batch"], kind)
    raw = np.ascontiguousarray(x.astype(np.complex64)).view(np.float32)
    assert hashlib.sha256(raw.tobytes()).hexdigest() == REF_INPUTS["sha256"][f"n{n}_k{kind}"]


@pytest.mark.skipif(not (oracle.HERE / "_ref" / "libthff_ref_inputs.so").exists(),
                    reason="reference input harness not built (oracle/build_ref.py)")
def test_validation_inputs_against_live_reference_generator():
    """Same check against the reference's generator itself, where
    oracle/build_ref.py has compiled it, at a batch other than the digests'."""
    import ctypes

    lib = ctypes.CDLL(str(oracle.HERE / "_ref" / "libthff_ref_inputs.so"))
    lib.thff_ref_make_input.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    for n in SIZES:
        for kind in range(4):
            out = np.zeros((5, n, 2), np.float32)
            lib.thff_ref_make_input(n, 5, kind, out.ctypes.data)
            ref = (out[..., 0] + 1j * out[..., 1]).astype(np.complex64)
            assert np.array_equal(oracle.make_validation_input(n, 5, kind), ref), (n, kind)


def test_circconv1d_matches_fft_convolution():
    x, h, y = GOLD["conv1d_x"], GOLD["conv1d_h"], GOLD["conv1d_y"]
    got = oracle.circconv1d(x, h)
    assert np.max(np.abs(got - y)) < 1e-10


def test_circconv2d_matches_fft_convolution():
    rng = np.random.default_rng(9)
    x = rng.standard_normal((3, 32, 16))
    f = rng.standard_normal((2, 5, 5))
    idx = np.array([0, 1, 1], dtype=np.int32)
    got = oracle.circconv2d(x, f, idx)
    for b in range(3):
        fp = np.zeros((32, 16))
        fp[:5, :5] = f[idx[b]]
        ref = np.real(np.fft.ifft2(np.fft.fft2(x[b]) * np.fft.fft2(fp)))
        assert np.max(np.abs(got[b] - ref)) < 1e-10


def test_paper_lcg_input_is_bounded():
    # sample/bench/paper_fft.cu:27-43: values in [-1, 1) / sqrt(n)
    x = oracle.make_paper_input(256, 8)
    assert np.abs(x.real).max() <= 1 / 16 and np.abs(x.imag).max() <= 1 / 16
    assert x[0, 0] != 0


REF_GPU = np.load(__import__("pathlib").Path(__file__).parent / "golden" / "ref_gpu_outputs.npz")


@pytest.mark.parametrize("key", sorted(REF_GPU.files))
def test_oracle_matches_reference_gpu_output(key):
    """The reference's ThunderFFT_global (include/thunderfft/detail/
    thunderfft_impl_kernel.cuh:6-41) on the validation's seeded Gaussian
    input (fft_validation.cu:130-163, batch 2) agrees with the FP64 oracle on
    the same input (rounded to the storage type) within the reference's own
    gate, relative L2 <= 5e-3 (fft_validation.cu:26): same sign convention,
    same unnormalised inverse, same element order.  Measured: TF32
    1.3e-3..2.7e-3, FP16 3.9e-4..6.3e-4."""
    T, n_s, d = key.split("_")
    n, fwd = int(n_s[1:]), d == "fwd"
    x = oracle.make_validation_input(n, 2, 0)
    a = REF_GPU[key]
    if T == "float":
        ref = a.astype(np.complex128)
        xin = x.astype(np.complex64).astype(np.complex128)
    else:
        ref = a[..., 0].astype(np.float64) + 1j * a[..., 1].astype(np.float64)
        xin = x.real.astype(np.float16).astype(np.float64) + 1j * x.imag.astype(np.float16).astype(np.float64)
    assert oracle.rel_l2(ref, oracle.fft(xin, fwd)) <= 5e-3, key
    # the comparison discriminates: the opposite direction is far outside the gate
    assert oracle.rel_l2(ref, oracle.fft(xin, not fwd)) > 0.5, key
