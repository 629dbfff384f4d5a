"""Build libthunderfft_b200.so (sm_100a) in-tree with nvcc.

The library is plain CUDA C++ behind the C ABI in include/thff.h; it links the
CUDA runtime statically so that the .so has no runtime search-path needs on a
GPU box.  Usage:  python -m thunderfft_b200.build  [--force]
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libthunderfft_b200.so"
SOURCES = [CSRC / "thff_capi.cu"]
DEPS = SOURCES + sorted(CSRC.glob("*.cuh")) + [ROOT / "include" / "thff.h"]

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or "/usr/local/cuda/bin/nvcc"
    return cand if Path(cand).exists() else "nvcc"


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    return all(d.stat().st_mtime <= t for d in DEPS if d.exists())


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH_FLAGS, "-std=c++17", "-O3", "-lineinfo", "-shared", "-Xcompiler", "-fPIC",
           "-cudart", "static", "-I", str(ROOT / "include"), "-o", str(tmp), *map(str, SOURCES)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("nvcc failed building libthunderfft_b200.so")
    if verbose:
        sys.stderr.write(res.stderr)
    os.replace(tmp, LIB)
    return LIB


PAPER_FFT_SRC = PKG / "bench" / "paper_fft.cu"
PAPER_FFT = PKG / "bench" / "thff_paper_fft"


def build_paper_fft(force: bool = False) -> Path:
    """The device-API timing CLI (bench/paper_fft.cu), linked like a C++ user
    of the library links it (header + -lthunderfft_b200, plus cuFFT for its
    accuracy check)."""
    lib = build()
    headers = [p for p in (ROOT / "include").rglob("*") if p.suffix in (".h", ".cuh", ".hpp")]
    if (not force and PAPER_FFT.exists() and
            all(p.stat().st_mtime <= PAPER_FFT.stat().st_mtime for p in [PAPER_FFT_SRC, lib, *headers])):
        return PAPER_FFT
    cmd = [nvcc(), *ARCH_FLAGS, "-std=c++17", "-O3", "-I", str(ROOT / "include"), str(PAPER_FFT_SRC), "-o",
           str(PAPER_FFT), "-L", str(lib.parent), "-lthunderfft_b200", "-lcufft", "-Xlinker", f"-rpath={lib.parent}"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("nvcc failed building thff_paper_fft")
    return PAPER_FFT


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
    if "--paper-fft" in sys.argv:
        print(build_paper_fft(force="--force" in sys.argv))
