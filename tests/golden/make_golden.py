"""Generate the committed golden fixtures in tests/golden/.

Inputs come from the reference validation's own seeded generators (restated
bit-exactly in oracle/thff_oracle.cpp: sample/validation/fft_validation.cu:130-163,
sample/fft1d/main.cu:63-77) and from BASELINE config 1 (N=64, batch 16,
U[-1,1) from a seed).  Expected outputs are computed with numpy's pocketfft in
FP64 — an implementation independent of the oracle — so the fixtures pin the
oracle as well as the CUDA path.

Run:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

import oracle  # noqa: E402


def half_repr(x: np.ndarray) -> np.ndarray:
    """Values actually represented after storing x as half2."""
    return (x.real.astype(np.float16).astype(np.float64) + 1j * x.imag.astype(np.float16).astype(np.float64))


def main() -> None:
    out = {}
    # N=64, batch 16, U[-1,1) re/im from seed 20260101
    rng = np.random.default_rng(20260101)
    x = (rng.uniform(-1, 1, (16, 64)) + 1j * rng.uniform(-1, 1, (16, 64))).astype(np.complex64)
    out["cfg1_x"] = x
    out["cfg1_fwd"] = np.fft.fft(x.astype(np.complex128), axis=-1)
    out["cfg1_inv"] = np.fft.ifft(x.astype(np.complex128), axis=-1) * 64
    # reference validation inputs (4 kinds), batch 2
    for n in (64, 256, 1024):
        for kind in range(4):
            xi = oracle.make_validation_input(n, 2, kind)
            out[f"val_n{n}_k{kind}_x"] = xi
            out[f"val_n{n}_k{kind}_fwd"] = np.fft.fft(xi.astype(np.complex128), axis=-1)
            out[f"val_n{n}_k{kind}_fwd_half"] = np.fft.fft(half_repr(xi), axis=-1)
    # quick-start tones (N=64, batch 16)
    xf = oracle.make_fft1d_input(16)
    out["fft1d_x"] = xf
    out["fft1d_fwd"] = np.fft.fft(xf.astype(np.complex128), axis=-1)
    # small real circular convolution (conv1d semantics), N=256, 9 taps
    rng = np.random.default_rng(5)
    xs = rng.standard_normal((3, 256))
    h = rng.standard_normal(9)
    hp = np.zeros(256)
    hp[:9] = h
    out["conv1d_x"] = xs
    out["conv1d_h"] = h
    out["conv1d_y"] = np.real(np.fft.ifft(np.fft.fft(xs, axis=-1) * np.fft.fft(hp)[None, :], axis=-1))
    np.savez_compressed(HERE / "golden_fft.npz", **out)
    print("wrote", HERE / "golden_fft.npz", len(out), "arrays")


if __name__ == "__main__":
    main()
