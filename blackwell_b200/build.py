"""Build recipe for the native library: nvcc, sm_100a, in-tree.

    python -m blackwell_b200.build        # -> blackwell_b200/libbw_attn.so

It also links the C++ harness ``bw_harness`` (harness/bw_harness.cpp) against
the library.  Every .cu under csrc/ is compiled with
``-gencode arch=compute_100a,code=sm_100a -lineinfo -O3`` and linked into one
shared library with the CUDA runtime linked statically (no torch types cross
the boundary; the library only depends on the driver at run time).
"""
from __future__ import annotations

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
OUT = HERE / "libbw_attn.so"
HARNESS = HERE / "bw_harness"
HARNESS_SRC = HERE / "harness" / "bw_harness.cpp"
BUILD = HERE / "_build"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-O3", "-std=c++17",
         "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr"]


def _sources():
    return sorted(CSRC.glob("*.cu"))


def _deps():
    return sorted(CSRC.glob("*.cu*")) + sorted(CSRC.glob("*.h")) + sorted((HERE.parent / "include").glob("*.h"))


def up_to_date() -> bool:
    if not OUT.exists() or not HARNESS.exists():
        return False
    t = min(OUT.stat().st_mtime, HARNESS.stat().st_mtime)
    return all(p.stat().st_mtime <= t for p in _deps() + [HARNESS_SRC])


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return OUT
    BUILD.mkdir(exist_ok=True)

    def compile_one(src: Path) -> Path:
        obj = BUILD / (src.stem + ".o")
        cmd = [NVCC, *FLAGS, "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
        return obj

    with ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as ex:
        objs = list(ex.map(compile_one, _sources()))
    tmp = OUT.with_suffix(".so.tmp")
    cmd = [NVCC, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-o", str(tmp), *map(str, objs)]
    subprocess.run(cmd, check=True)
    os.replace(tmp, OUT)
    build_harness(verbose)
    return OUT


def build_harness(verbose: bool = False) -> Path:
    """The C++ harness (reference-style main over the C ABI), linked to the library."""
    cmd = [NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-I", str(HERE.parent / "include"),
           str(HARNESS_SRC), "-o", str(HARNESS),
           "-L", str(HERE), "-lbw_attn", "-Xlinker", "-rpath,$ORIGIN"]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    return HARNESS


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
