"""Build recipe for oracle/_ref/ — TEST INFRASTRUCTURE ONLY.

Compiles, for sm_100a with nvcc directly (the reference's CMake build is not
used), from the reference sources where they lie (read-only; the directory is
THFF_REFERENCE_DIR when set, else the build container's reference checkout):
  libthff_ref.so        oracle/ref_harness.cu against the reference headers
                        (its ThunderFFT_global, for parity and GPU timing);
  ref_conv1d_tiled      the reference's tiled conv1d sample as it is
                        (sample/conv1d/main.cu);
  ref_conv1d_full       the reference's fused FFT-conv sample as it is
                        (sample/conv1d/conv1d_fullfft_l4096_thunder.cu);
  ref_paper_fft         the reference's device-API timing CLI
                        (sample/bench/paper_fft.cu, with its util/ and
                        baseline/ include directories and --use_fast_math,
                        as its CMakeLists builds it).
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
REF = Path(os.environ.get("THFF_REFERENCE_DIR", "/root/reference"))
REF_INCLUDE = REF / "include"
OUT = HERE / "_ref" / "libthff_ref.so"

SAMPLES = {
    "ref_conv1d_tiled": REF / "sample" / "conv1d" / "main.cu",
    "ref_conv1d_full": REF / "sample" / "conv1d" / "conv1d_fullfft_l4096_thunder.cu",
    "ref_paper_fft": REF / "sample" / "bench" / "paper_fft.cu",
}
EXTRA_FLAGS = {
    "ref_paper_fft": ["-I", str(REF / "sample" / "bench" / "util"), "-I", str(REF / "sample" / "bench" / "baseline"),
                      "--use_fast_math"],
}
NVCC = "/usr/local/cuda/bin/nvcc"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def build_sample(name: str, src: Path) -> None:
    out = HERE / "_ref" / name
    if out.exists() and out.stat().st_mtime >= src.stat().st_mtime:
        return
    tmp = out.with_suffix(".tmp")
    subprocess.run([NVCC, "-std=c++17", "-O3", *ARCH, "-I", str(REF_INCLUDE), *EXTRA_FLAGS.get(name, []), str(src),
                    "-lcufft", "-o", str(tmp)], check=True)
    tmp.replace(out)
    print(out)


def main() -> int:
    if not REF_INCLUDE.exists():
        print("reference sources not present; nothing to build")
        return 0
    src = HERE / "ref_harness.cu"
    OUT.parent.mkdir(exist_ok=True)
    if not (OUT.exists() and OUT.stat().st_mtime >= src.stat().st_mtime):
        tmp = OUT.with_suffix(".so.tmp")
        cmd = [NVCC, "-std=c++17", "-O3", *ARCH, "-shared", "-Xcompiler", "-fPIC,-fvisibility=hidden",
               "-cudart", "static", "-I", str(REF_INCLUDE), str(src), "-o", str(tmp)]
        subprocess.run(cmd, check=True)
        tmp.replace(OUT)
        print(OUT)
    for name, sample in SAMPLES.items():
        if sample.exists():
            build_sample(name, sample)
    return 0


if __name__ == "__main__":
    sys.exit(main())
