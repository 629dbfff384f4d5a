"""Freeze the reference's own GPU output as committed fixtures.

Runs the REFERENCE's ThunderFFT_global (recompiled for sm_100a from its own
headers into oracle/_ref/libthff_ref.so by oracle/build_ref.py) on the
reference validation's seeded Gaussian input (batch 2) for N in
{64, 256, 1024, 4096}, float and half, both directions, and stores the
outputs in tests/golden/ref_gpu_outputs.npz.  Inputs are regenerated at test
time from the bit-exact generator restatement, so only outputs are stored.
Needs a B200:  python tests/golden/make_ref_gpu_golden.py [OUT.npz]
"""
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))
import oracle  # noqa: E402

SIZES = (64, 256, 1024, 4096)


def main(out: Path) -> None:
    res = {}
    for T in ("float", "half"):
        for n in SIZES:
            x = oracle.make_validation_input(n, 2, 0)
            if T == "float":
                din = torch.from_numpy(np.ascontiguousarray(x)).cuda()
            else:
                din = torch.from_numpy(np.stack([x.real, x.imag], -1).astype(np.float16)).cuda()
            for fwd in (True, False):
                dout = torch.empty_like(din)
                oracle.ref_global(T, n, fwd, din.data_ptr(), dout.data_ptr(), 2)
                torch.cuda.synchronize()
                res[f"{T}_n{n}_{'fwd' if fwd else 'inv'}"] = dout.cpu().numpy()
    np.savez_compressed(out, **res)
    print("wrote", out)


if __name__ == "__main__":
    main(Path(sys.argv[1]) if len(sys.argv) > 1 else HERE / "ref_gpu_outputs.npz")
