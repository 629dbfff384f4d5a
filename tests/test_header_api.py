"""The C++ header API used the way a reference user uses it
(include/thunderfft/thunderfft.cuh compiled into a user program and linked
with libthunderfft_b200.so): host contract (no GPU), device-API composition
and twiddle-cache lifecycle (GPU)."""
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

import oracle

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE / "cpp"))
import build as cppbuild  # noqa: E402


def test_host_contract_program_without_gpu():
    exe = cppbuild.build("host_contract")
    res = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120,
                         env={"CUDA_VISIBLE_DEVICES": "", "PATH": "/usr/bin:/bin"})
    assert res.returncode == 0, res.stderr
    assert "18 checks passed" in res.stdout


@pytest.mark.gpu
def test_device_api_composition(cuda, tmp_path):
    exe = cppbuild.build("device_api")
    res = subprocess.run([str(exe), str(tmp_path)], capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stdout + res.stderr
    files = sorted(tmp_path.glob("devapi_*.bin"))
    assert len(files) == 28
    for f in files:
        raw = f.read_bytes()
        n, batch, guard_bad, _ = np.frombuffer(raw[:16], dtype=np.int32)
        data = np.frombuffer(raw[16:], dtype=np.complex64).reshape(3, batch, n)
        x, y, y2 = data.astype(np.complex128)
        forward = f.stem.endswith("fwd")
        ref = oracle.fft(x, forward)
        assert guard_bad == 0, f.name
        assert np.isfinite(y).all() and np.isfinite(y2).all(), f.name
        e1, e2 = oracle.rel_l2(y, ref), oracle.rel_l2(y2, ref)
        # the reference's gate for both types; float N <= 256 runs TF32 warp
        # MMAs (the reference's arithmetic), the larger float sizes FP32
        # arithmetic, which also meets a 1e-5 gate
        gate = 1e-5 if ("_float_" in f.name and n > 256) else 5e-3
        assert e1 <= gate and e2 <= gate, (f.name, e1, e2)


@pytest.mark.gpu
def test_cache_lifecycle_program(cuda):
    exe = cppbuild.build("cache_lifecycle")
    res = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stdout + res.stderr
    assert "checks passed" in res.stdout


@pytest.mark.gpu
def test_cuda_error_contract_program(cuda):
    """A CUDA failure inside the header API throws std::runtime_error with the
    reference's "[ThunderFFT] <what>: <cudaGetErrorString>" message and leaves
    the library usable (failure injected on the host, no GPU fault)."""
    exe = cppbuild.build("cuda_error_contract")
    res = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stdout + res.stderr
    assert "checks passed" in res.stdout
