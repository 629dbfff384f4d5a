"""Freeze the reference validation program's own seeded inputs as digests.

Calls the REFERENCE's make_input (sample/validation/fft_validation.cu:130-163),
compiled from its source by oracle/build_ref.py into
oracle/_ref/libthff_ref_inputs.so, for every size and input kind at the
program's default batch (64), and records the SHA-256 of each array
(complex64, interleaved re/im, signal-major) in tests/golden/ref_inputs.json.
tests/test_oracle.py then checks that the oracle's restatement reproduces
every array bit for bit, on any machine, without the reference present.
Run in the build container:  python tests/golden/make_ref_inputs.py
"""
from __future__ import annotations

import ctypes
import hashlib
import json
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE.parents[1] / "oracle" / "_ref" / "libthff_ref_inputs.so"
SIZES = (64, 128, 256, 512, 1024, 2048, 4096)
BATCH = 64   # the validation program's default batch (fft_validation.cu:168)


def main() -> None:
    lib = ctypes.CDLL(str(LIB))
    lib.thff_ref_make_input.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    digests = {}
    for n in SIZES:
        for kind in range(4):
            out = np.zeros((BATCH, n, 2), np.float32)
            lib.thff_ref_make_input(n, BATCH, kind, out.ctypes.data)
            digests[f"n{n}_k{kind}"] = hashlib.sha256(out.tobytes()).hexdigest()
    path = HERE / "ref_inputs.json"
    path.write_text(json.dumps({"source": "sample/validation/fft_validation.cu:130-163 make_input",
                                "batch": BATCH, "layout": "complex64 [batch][n] interleaved",
                                "sha256": digests}, indent=1) + "\n")
    print("wrote", path, len(digests), "digests")


if __name__ == "__main__":
    main()
