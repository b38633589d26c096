"""Builds the reference's own split-length GQA kernel program (TEST INFRASTRUCTURE ONLY).

The reference's `gqa_split` path is `launch_gqa_v1` in
src/SM120/attention/adhitya_GQA.cu:199-213 (kernel :63-188, harness main()
:215-325, with the header-only utilities include/utils/kernelUtils.cuh and
kernelBench.cuh).  It is plain CUDA C++ that compiles from those few files, so
this recipe compiles it, unmodified and where it lies in the reference tree,
into ``oracle/_ref/adhitya_gqa`` (git-ignored; it travels to the GPU box with
the other built files).  Its main() runs the kernel at B=16, Hq=12, Hkv=4,
Sq=4096, Skv=2048, D=64, compares O and LSE with ``data/gqa_split_*.bin``
(atol = rtol = 2e-2) when those files exist in its working directory, and
times the kernel with the reference's own harness (25 warm-ups, 100 timed
runs, 256 MiB L2 flush per run).  ``tests/test_reference_kernel_gpu.py``
uses it as a cross-check and a timing comparator.

The reference's tcgen05 kernels (src/SM103) cannot be built here: nvcc 12.9
rejects their > 48 KB static shared memory.
"""
from __future__ import annotations

import os
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref" / "adhitya_gqa"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")


def default_reference_root() -> Path:
    """The reference checkout next to this repository, if any."""
    return HERE.parent.parent / "reference"


def build(reference_root: Path | None = None, verbose: bool = False) -> Path | None:
    """Compile the reference program; returns its path, or None when the
    reference tree is not present (the GPU box only uses the prebuilt file)."""
    root = Path(reference_root) if reference_root else default_reference_root()
    src = root / "src" / "SM120" / "attention" / "adhitya_GQA.cu"
    inc = root / "include"
    if not src.is_file() or not (inc / "utils" / "kernelBench.cuh").is_file():
        return None
    if OUT.exists() and OUT.stat().st_mtime >= src.stat().st_mtime:
        return OUT
    OUT.parent.mkdir(exist_ok=True)
    cmd = [NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", f"-I{inc}", str(src),
           "-o", str(OUT)]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    return OUT


if __name__ == "__main__":
    print(build(verbose=True))
