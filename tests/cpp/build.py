"""Build the C++ programs under tests/cpp against the public header and
libthunderfft_b200.so (the way a C++ user of the library links it).
Binaries go to tests/cpp/_build/ (git-ignored; they travel to GPU boxes)."""
from __future__ import annotations

import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
OUT = HERE / "_build"
PROGRAMS = ("host_contract", "device_api", "cache_lifecycle", "cuda_error_contract")


def build(name: str, force: bool = False) -> Path:
    sys.path.insert(0, str(ROOT))
    from thunderfft_b200 import build as libbuild

    lib = libbuild.build()
    src = HERE / f"{name}.cu"
    exe = OUT / name
    headers = [p for p in (ROOT / "include").rglob("*") if p.suffix in (".h", ".cuh", ".hpp")]
    if not force and exe.exists() and all(p.stat().st_mtime <= exe.stat().st_mtime for p in [src, lib, *headers]):
        return exe
    OUT.mkdir(exist_ok=True)
    cmd = [libbuild.nvcc(), "-std=c++17", "-O2", *libbuild.ARCH_FLAGS, "-I", str(ROOT / "include"), str(src),
           "-o", str(exe), "-L", str(lib.parent), "-lthunderfft_b200", "-Xlinker", f"-rpath={lib.parent}"]
    subprocess.run(cmd, check=True)
    return exe


def build_all(force: bool = False) -> None:
    for p in PROGRAMS:
        build(p, force)


if __name__ == "__main__":
    build_all("--force" in sys.argv)
