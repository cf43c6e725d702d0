"""Build the sm_100a shared library ``minicpm_b200/_lib/libminicpm_b200.so`` in place.

    python build.py            # from this directory, or call build() from Python

One nvcc invocation over ``csrc/b200_lib.cu`` (the kernels are headers it
includes), for ``-gencode arch=compute_100a,code=sm_100a`` only, with the
CUDA runtime linked statically so the library does not depend on which
libcudart the host process loaded first.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parent
SRC = HERE / "csrc" / "b200_lib.cu"
OUT = HERE / "minicpm_b200" / "_lib" / "libminicpm_b200.so"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-shared", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-cudart", "static",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def sources() -> list[Path]:
    return sorted((HERE / "csrc").glob("*.cu*")) + [REPO / "include" / "minicpm_b200.h"]


def up_to_date() -> bool:
    if not OUT.exists():
        return False
    mtime = OUT.stat().st_mtime
    return all(p.stat().st_mtime <= mtime for p in sources() + [Path(__file__)])


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> Path:
    if not force and up_to_date():
        return OUT
    OUT.parent.mkdir(parents=True, exist_ok=True)
    tmp = OUT.with_suffix(".so.tmp")
    cmd = [nvcc(), *NVCC_FLAGS, *(extra or []), "-I", str(REPO / "include"), "-I", str(HERE / "csrc"),
           str(SRC), "-o", str(tmp)]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout or res.stderr):
        print(res.stdout + res.stderr, flush=True)
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    extra = [a for a in sys.argv[1:] if a not in ("-f", "--force", "-v")]
    build(force=True, verbose="-v" in sys.argv, extra=extra)
    print(OUT)
