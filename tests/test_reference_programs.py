"""The reference's own test programs, compiled unchanged against this library.

oracle/build_ref.py compiles sample/validation/fft_validation.cu,
sample/validation/cache_validation.cu and sample/fft1d/main.cu from the
reference's sources with this repository's include/ on the include path and
libthunderfft_b200.so linked in place of the reference's header-only kernels
(oracle/_ref/refval_*).  They exercise the public surface a user of the
reference calls:

* fft_validation: the 18 host-side argument checks (--host-only, no CUDA),
  then every N in 64..4096, float/TF32 and half/FP16, both directions, the
  device-routine composition validate_core (bench_layout tiles,
  make_reg_b_precompute, ThunderFFT_kernel_reg, the movement helpers, shared
  memory guards) and the public ThunderFFT_global with partial batches, on
  the four seeded input kinds, against cuFFT Z2Z in FP64
  (fft_validation.cu:83-123,180-266,278-311,331-352);
* cache_validation: twiddle cache lifecycle, the test-visible device symbols
  and per-device ownership (cache_validation.cu:104-148);
* fft1d: the quick-start example against cuFFT (fft1d/main.cu:90-178).

A program's exit status is its verdict (0 = every case passed).
"""
import os
import subprocess
from pathlib import Path

import pytest

REF = Path(__file__).resolve().parents[1] / "oracle" / "_ref"
FFT_VALIDATION = REF / "refval_fft_validation"
CACHE_VALIDATION = REF / "refval_cache_validation"
FFT1D = REF / "refval_fft1d"


def run(cmd, timeout=900):
    env = dict(os.environ)
    return subprocess.run([str(c) for c in cmd], capture_output=True, text=True, timeout=timeout, env=env)


@pytest.mark.skipif(not FFT_VALIDATION.exists(), reason="reference programs not built (oracle/build_ref.py)")
def test_reference_host_checks_unchanged():
    """fft_validation.cu --host-only: the reference's 18 argument checks
    (negative batch, null and aliased pointers, zero batch without CUDA, bad
    initialization lengths for both types) pass against this library's
    header, before any CUDA call."""
    res = run([FFT_VALIDATION, "--host-only"], timeout=120)
    assert res.returncode == 0, res.stdout + res.stderr
    assert "18 checks passed" in res.stderr


@pytest.mark.gpu
@pytest.mark.skipif(not FFT_VALIDATION.exists(), reason="reference programs not built (oracle/build_ref.py)")
def test_reference_fft_validation_full_matrix(cuda, tmp_path):
    """The full validation matrix of the reference's own program: 7 sizes x
    2 types x 2 directions x {device-routine composition, public wrapper} x
    4 input kinds, plus partial batches {1, BPB-1, BPB+1} through the public
    wrapper; every case must keep relative L2 <= 5e-3 against cuFFT Z2Z,
    finite outputs and untouched memory guards."""
    csv = tmp_path / "validation.csv"
    res = run([FFT_VALIDATION, "--csv", csv])
    assert res.returncode == 0, res.stderr + res.stdout[-4000:]
    rows = csv.read_text().strip().splitlines()
    header, cases = rows[0].split(","), [r.split(",") for r in rows[1:]]
    assert len(cases) >= 7 * 2 * 4 * 4
    col = {name: i for i, name in enumerate(header)}
    assert all(c[col["pass"]] == "1" for c in cases)
    assert {c[col["path"]] for c in cases} == {"direct_core_guarded", "public_global"}
    assert {int(c[col["N"]]) for c in cases} == {64, 128, 256, 512, 1024, 2048, 4096}
    worst = max(float(c[col["relative_l2"]]) for c in cases)
    assert worst <= 5e-3
    print(f"{len(cases)} cases passed; worst relative L2 {worst:.3e}")


@pytest.mark.gpu
@pytest.mark.skipif(not CACHE_VALIDATION.exists(), reason="reference programs not built (oracle/build_ref.py)")
def test_reference_cache_validation(cuda):
    """The reference's twiddle-cache lifecycle program: W[0] = 1, W[1] of the
    current length, the FP16 unit table equal to its host builder, same-length
    cache hits keep the allocation, another length replaces it, Finalize
    clears the symbols, repeated Finalize is harmless, and each visible
    device keeps its own cache."""
    res = run([CACHE_VALIDATION], timeout=300)
    assert res.returncode == 0, res.stderr + res.stdout[-4000:]
    assert "checks passed" in res.stderr


@pytest.mark.gpu
@pytest.mark.skipif(not FFT1D.exists(), reason="reference programs not built (oracle/build_ref.py)")
@pytest.mark.parametrize("batch", [16, 4096])
def test_reference_fft1d_example(cuda, batch):
    """The reference's quick-start example: float N = 64 forward through
    ThunderFFT_global against cuFFT, relative L2 and Linf <= 5e-3."""
    res = run([FFT1D, batch], timeout=300)
    assert res.returncode == 0, res.stderr + res.stdout
    assert "PASS" in res.stdout
