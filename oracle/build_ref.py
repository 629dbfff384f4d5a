"""Build recipe for oracle/_ref/libthff_ref.so — TEST INFRASTRUCTURE ONLY.

Compiles oracle/ref_harness.cu against the reference's own headers where they
lie (/root/reference/include, read-only) for sm_100a with nvcc directly (the
reference's CMake build is not used).  Output goes only to oracle/_ref/.
Run in the build container:  python oracle/build_ref.py
"""
from __future__ import annotations

import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REF_INCLUDE = Path("/root/reference/include")
OUT = HERE / "_ref" / "libthff_ref.so"


def main() -> int:
    if not REF_INCLUDE.exists():
        print("reference sources not present; nothing to build")
        return 0
    src = HERE / "ref_harness.cu"
    if OUT.exists() and OUT.stat().st_mtime >= src.stat().st_mtime:
        return 0
    OUT.parent.mkdir(exist_ok=True)
    tmp = OUT.with_suffix(".so.tmp")
    cmd = ["/usr/local/cuda/bin/nvcc", "-std=c++17", "-O3", "-gencode", "arch=compute_100a,code=sm_100a",
           "-shared", "-Xcompiler", "-fPIC,-fvisibility=hidden", "-cudart", "static", "-I", str(REF_INCLUDE),
           str(src), "-o", str(tmp)]
    subprocess.run(cmd, check=True)
    tmp.replace(OUT)
    print(OUT)
    return 0


if __name__ == "__main__":
    sys.exit(main())
