"""Builds the reference's own SM120 attention programs (TEST INFRASTRUCTURE ONLY).

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

The reference's non-causal GQA program (src/SM120/attention/GQA_sm120.cu:
`gqa_v1` two-pass :58-184 and `gqa_v2` online softmax :187-345, main()
:383-518) goes to ``oracle/_ref/gqa_sm120``: B=16, Hq=12, Hkv=4, S=4096,
D=64, checked against ``data/gqa_*.bin`` the same way.

Likewise the reference's fp32 MHA program (src/SM120/attention/MHA_sm120.cu:
`mha_v3_tc`, 3xTF32 split, :64-170, launch and main() :289-370) goes to
``oracle/_ref/mha_sm120``, with its data directory (a compile-time macro,
MHA_DATA_DIR) set to ``data`` relative to its working directory; main() runs
B=16, H=12, S=1024, D=64, reports the precision of its output and of the
files' "SDPA" output against the files' fp64 output, and times the kernel.

The reference's fused QK-norm + RoPE + attention program
(src/SM103/attention/GQA_fused_sm103.cu) is WMMA code and compiles for sm_100a.
Its ground truth for the fused op is two naive GPU kernels, ``ref_norm_rope``
and ``ref_attention`` (:328-420); ``oracle/ref_fused_driver.cu`` includes that
file unmodified (its main() renamed) and runs those two kernels on inputs given
in files, into ``oracle/_ref/ref_fused`` (used by
``tests/test_norm_rope_ref_gpu.py`` to pin the fused op).

The reference's tcgen05 kernels (src/SM103, GQA_sm103*.cu) cannot be built
here: nvcc 12.9 rejects their > 48 KB static shared memory.
"""
from __future__ import annotations

import os
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref" / "adhitya_gqa"
OUT_MHA = HERE / "_ref" / "mha_sm120"
OUT_GQA = HERE / "_ref" / "gqa_sm120"
OUT_FUSED = HERE / "_ref" / "ref_fused"
FUSED_DRIVER = HERE / "ref_fused_driver.cu"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")


def default_reference_root() -> Path:
    """The reference checkout next to this repository, if any."""
    return HERE.parent.parent / "reference"


def _compile(src: Path, inc: Path, out: Path, extra: list[str], verbose: bool, deps=()) -> Path:
    if out.exists() and all(out.stat().st_mtime >= p.stat().st_mtime for p in (src, *deps)):
        return out
    out.parent.mkdir(exist_ok=True)
    cmd = [NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", f"-I{inc}", *extra, str(src),
           "-o", str(out)]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    return out


def build(reference_root: Path | None = None, verbose: bool = False) -> list[Path]:
    """Compile the reference programs; returns their paths (empty when the
    reference tree is not present: the GPU box only uses the prebuilt files)."""
    root = Path(reference_root) if reference_root else default_reference_root()
    att = root / "src" / "SM120" / "attention"
    inc = root / "include"
    if not (inc / "utils" / "kernelBench.cuh").is_file():
        return []
    built = []
    if (att / "adhitya_GQA.cu").is_file():
        built.append(_compile(att / "adhitya_GQA.cu", inc, OUT, [], verbose))
    if (att / "GQA_sm120.cu").is_file():
        built.append(_compile(att / "GQA_sm120.cu", inc, OUT_GQA, [], verbose))
    if (att / "MHA_sm120.cu").is_file():
        built.append(_compile(att / "MHA_sm120.cu", inc, OUT_MHA, ["-DMHA_DATA_DIR=data"], verbose))
    fused = root / "src" / "SM103" / "attention" / "GQA_fused_sm103.cu"
    if fused.is_file():
        built.append(_compile(FUSED_DRIVER, inc, OUT_FUSED, [f"-I{fused.parent}"], verbose, deps=(fused,)))
    return built


if __name__ == "__main__":
    print(build(verbose=True))
