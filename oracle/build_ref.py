"""Build recipe for oracle/_ref/ — TEST INFRASTRUCTURE ONLY.

Compiles, for sm_100a with nvcc directly (the reference's CMake build is not
used), from the reference sources where they lie (read-only; the directory is
THFF_REFERENCE_DIR when set, else the build container's reference checkout).

Against the REFERENCE's own headers (the reference as it is):
  libthff_ref.so          oracle/ref_harness.cu: its ThunderFFT_global, for
                          parity and GPU timing;
  libthff_ref_inputs.so   oracle/ref_inputs.cu: its validation program's
                          seeded input generator (make_input), to pin the
                          oracle's restatement bit for bit (PTX only: no
                          kernel of it is launched);
  ref_conv1d_tiled        the tiled conv1d sample (sample/conv1d/main.cu);
  ref_conv1d_full         the fused FFT-conv sample
                          (sample/conv1d/conv1d_fullfft_l4096_thunder.cu);
  ref_conv1d_io           oracle/ref_conv1d_io.cu: that sample's fused kernel
                          run on inputs read from a file, for parity of the
                          conv1d on identical signals and taps;
  ref_paper_fft           the device-API timing CLI (sample/bench/paper_fft.cu,
                          with its util/ and baseline/ include directories and
                          --use_fast_math, as its CMakeLists builds it).

Against THIS library (include/ of this repository and
thunderfft_b200/libthunderfft_b200.so), the reference's own test programs
compiled unchanged, which is the drop-in check of the public surface:
  refval_fft_validation   sample/validation/fft_validation.cu (all sizes,
                          both types, both directions, the device routine
                          composition and the public wrapper, against cuFFT
                          Z2Z; --host-only runs its 18 argument checks);
  refval_cache_validation sample/validation/cache_validation.cu (twiddle
                          cache lifecycle and device ownership);
  refval_fft1d            sample/fft1d/main.cu (quick-start example against
                          cuFFT).

The samples link cuFFT (they use it for filter spectra or accuracy checks).
Output goes only to oracle/_ref/.  Run in the build container:
    python oracle/build_ref.py
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
REF = Path(os.environ.get("THFF_REFERENCE_DIR", "/root/reference"))
REF_INCLUDE = REF / "include"
OUT_DIR = HERE / "_ref"
OUT = OUT_DIR / "libthff_ref.so"
OUT_INPUTS = OUT_DIR / "libthff_ref_inputs.so"
VALIDATION_SRC = REF / "sample" / "validation" / "fft_validation.cu"
CONV1D_SRC = REF / "sample" / "conv1d" / "conv1d_fullfft_l4096_thunder.cu"

SAMPLES = {
    "ref_conv1d_tiled": REF / "sample" / "conv1d" / "main.cu",
    "ref_conv1d_full": CONV1D_SRC,
    "ref_paper_fft": REF / "sample" / "bench" / "paper_fft.cu",
}
EXTRA_FLAGS = {
    "ref_paper_fft": ["-I", str(REF / "sample" / "bench" / "util"), "-I", str(REF / "sample" / "bench" / "baseline"),
                      "--use_fast_math"],
}
# reference programs built against this library (name -> source, libraries)
REFVAL = {
    "refval_fft_validation": (VALIDATION_SRC, ["-lcufft"]),
    "refval_cache_validation": (REF / "sample" / "validation" / "cache_validation.cu", []),
    "refval_fft1d": (REF / "sample" / "fft1d" / "main.cu", ["-lcufft"]),
}
NVCC = "/usr/local/cuda/bin/nvcc"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def stale(out: Path, *deps: Path) -> bool:
    return not out.exists() or any(d.exists() and d.stat().st_mtime > out.stat().st_mtime for d in deps)


def build_sample(name: str, src: Path) -> None:
    out = OUT_DIR / name
    if not stale(out, src):
        return
    tmp = out.with_suffix(".tmp")
    subprocess.run([NVCC, "-std=c++17", "-O3", *ARCH, "-I", str(REF_INCLUDE), *EXTRA_FLAGS.get(name, []), str(src),
                    "-lcufft", "-o", str(tmp)], check=True)
    tmp.replace(out)
    print(out)


def build_refval(name: str, src: Path, libs: list[str]) -> None:
    """A reference test program, unchanged, against this repository's
    include/ and libthunderfft_b200.so (found through $ORIGIN at run time, so
    the binary works wherever the repository is copied)."""
    sys.path.insert(0, str(ROOT))
    from thunderfft_b200 import build as lib_build

    lib = lib_build.build()
    out = OUT_DIR / name
    headers = [p for p in (ROOT / "include").rglob("*") if p.is_file()]
    if not stale(out, src, lib, *headers):
        return
    tmp = out.with_suffix(".tmp")
    subprocess.run([NVCC, "-std=c++17", "-O3", *ARCH, "-I", str(ROOT / "include"), str(src), "-o", str(tmp),
                    "-L", str(lib.parent), "-lthunderfft_b200", *libs,
                    "-Xlinker", "-rpath=$ORIGIN/../../thunderfft_b200"], check=True)
    tmp.replace(out)
    print(out)


def main() -> int:
    if not REF_INCLUDE.exists():
        print("reference sources not present; nothing to build")
        return 0
    OUT_DIR.mkdir(exist_ok=True)
    src = HERE / "ref_harness.cu"
    if stale(OUT, src):
        tmp = OUT.with_suffix(".so.tmp")
        cmd = [NVCC, "-std=c++17", "-O3", *ARCH, "-shared", "-Xcompiler", "-fPIC,-fvisibility=hidden",
               "-cudart", "static", "-I", str(REF_INCLUDE), str(src), "-o", str(tmp)]
        subprocess.run(cmd, check=True)
        tmp.replace(OUT)
        print(OUT)
    src = HERE / "ref_inputs.cu"
    if VALIDATION_SRC.exists() and stale(OUT_INPUTS, src, VALIDATION_SRC):
        tmp = OUT_INPUTS.with_suffix(".so.tmp")
        cmd = [NVCC, "-std=c++17", "-O3", "-gencode", "arch=compute_100a,code=compute_100a", "-shared",
               "-Xcompiler", "-fPIC,-fvisibility=hidden", "-cudart", "static", "-I", str(REF_INCLUDE),
               f'-DTHFF_REF_VALIDATION_SOURCE="{VALIDATION_SRC}"', str(src), "-lcufft", "-o", str(tmp)]
        subprocess.run(cmd, check=True)
        tmp.replace(OUT_INPUTS)
        print(OUT_INPUTS)
    for name, sample in SAMPLES.items():
        if sample.exists():
            build_sample(name, sample)
    src, out = HERE / "ref_conv1d_io.cu", OUT_DIR / "ref_conv1d_io"
    if CONV1D_SRC.exists() and stale(out, src, CONV1D_SRC):
        tmp = out.with_suffix(".tmp")
        subprocess.run([NVCC, "-std=c++17", "-O3", *ARCH, "-I", str(REF_INCLUDE), "-I", str(CONV1D_SRC.parent),
                        f'-DTHFF_REF_CONV1D_SOURCE="{CONV1D_SRC}"', str(src), "-lcufft", "-o", str(tmp)], check=True)
        tmp.replace(out)
        print(out)
    for name, (sample, libs) in REFVAL.items():
        if sample.exists():
            build_refval(name, sample, libs)
    return 0


if __name__ == "__main__":
    sys.exit(main())
