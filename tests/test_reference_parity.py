"""Parity with the reference's own GPU output on the same inputs.

* against frozen reference outputs (tests/golden/ref_gpu_outputs.npz, made by
  tests/golden/make_ref_gpu_golden.py from the reference recompiled for
  sm_100a), always;
* against the live reference (oracle/_ref/libthff_ref.so) across the full
  matrix when that library is present.
Gate: relative L2 <= 5e-3 between this library's and the reference's output
(the reference's own gate, sample/validation/fft_validation.cu:26).
"""
from pathlib import Path

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).parent / "golden" / "ref_gpu_outputs.npz"
SIZES = (64, 128, 256, 512, 1024, 2048, 4096)


def as_complex(a, T):
    a = np.asarray(a)
    if T == "float":
        return a.astype(np.complex128)
    return a[..., 0].astype(np.float64) + 1j * a[..., 1].astype(np.float64)


def upload(x, T, torch):
    if T == "float":
        return torch.from_numpy(np.ascontiguousarray(x.astype(np.complex64))).cuda()
    return torch.from_numpy(np.stack([x.real, x.imag], -1).astype(np.float16)).cuda()


@pytest.mark.skipif(not GOLD.exists(), reason="frozen reference outputs not generated yet")
def test_against_frozen_reference_outputs(cuda):
    import torch

    import thunderfft_b200 as tf

    gold = np.load(GOLD)
    for key in gold.files:
        T, n_s, d = key.split("_")
        n, fwd = int(n_s[1:]), d == "fwd"
        x = oracle.make_validation_input(n, 2, 0)
        din = upload(x, T, torch)
        dout = torch.empty_like(din)
        tf.ThunderFFT_global(T, n, fwd, din, dout, 2)
        ours = as_complex(dout.cpu().numpy(), T)
        ref = as_complex(gold[key], T)
        assert oracle.rel_l2(ours, ref) <= 5e-3, key


@pytest.mark.skipif(not oracle.ref_available(), reason="reference harness not built (oracle/build_ref.py)")
@pytest.mark.parametrize("T", ["float", "half"])
@pytest.mark.parametrize("n", SIZES)
def test_against_live_reference(cuda, T, n):
    import torch

    import thunderfft_b200 as tf

    for kind in range(4):
        for batch in (64, 3):
            x = oracle.make_validation_input(n, batch, kind)
            din = upload(x, T, torch)
            for fwd in (True, False):
                dref, dours = torch.empty_like(din), torch.empty_like(din)
                oracle.ref_global(T, n, fwd, din.data_ptr(), dref.data_ptr(), batch)
                tf.ThunderFFT_global(T, n, fwd, din, dours, batch)
                ref, ours = as_complex(dref.cpu().numpy(), T), as_complex(dours.cpu().numpy(), T)
                assert oracle.rel_l2(ours, ref) <= 5e-3, (T, n, kind, batch, fwd)
