"""Interop with the reference's golden-file format.

The reference's Python scripts write every tensor as raw little-endian float32
with no header (`tensor.float().cpu().numpy().tofile(path)`,
base/baseline_gqa.py:165-170) and its CUDA harnesses read them back with
`loadBin(path, buf, n)` (include/utils/kernelUtils.cuh:191-199), narrowing
Q/K/V to bf16.  These helpers read and write that format so the reference's
`data/` directory can drive this library and this library's outputs can be
checked by the reference's harnesses.
"""
from __future__ import annotations

import math
from pathlib import Path

import numpy as np
import torch

# File stems and shapes the reference's generators write, per case.
# shapes use the generator's module constants (B, Hq, Hkv, S / Sq / Skv, D).
CASES = {
    "gqa": dict(prefix="gqa", causal=False, split=False),                 # base/baseline_gqa.py
    "gqa_causal": dict(prefix="gqa_causal", causal=True, split=False),    # base/baseline_gqa_causal.py
    "gqa_split": dict(prefix="gqa_split", causal=False, split=True),      # base/baseline_gqa_split.py
}


def load_bin(path, shape) -> np.ndarray:
    """Read a headerless float32 file and check its element count."""
    n = int(np.prod(shape))
    a = np.fromfile(path, dtype="<f4")
    if a.size != n:
        raise ValueError(f"{path}: expected {n} float32 values, found {a.size}")
    return a.reshape(shape)


def save_bin(path, array) -> None:
    """Write float32 values without a header (the reference's `.tofile` format)."""
    np.ascontiguousarray(np.asarray(array, dtype="<f4")).tofile(path)


def run_case(data_dir, case, B, Hq, Hkv, D, S=None, Sq=None, Skv=None, write_outputs=True):
    """Run this library on the reference's golden files of `case` in `data_dir`
    and return max-abs errors of O (vs the saved bf16 SDPA output) and LSE (vs the
    saved fp64 LSE).  Writes `<prefix>_o_bw.bin` / `<prefix>_lse_bw.bin` next to them."""
    from . import attention
    spec = CASES[case]
    pre = Path(data_dir) / spec["prefix"]
    Sq = Sq or S
    Skv = Skv or S
    q = torch.from_numpy(load_bin(f"{pre}_q.bin", (B, Hq, Sq, D))).bfloat16().cuda()
    k = torch.from_numpy(load_bin(f"{pre}_k.bin", (B, Hkv, Skv, D))).bfloat16().cuda()
    v = torch.from_numpy(load_bin(f"{pre}_v.bin", (B, Hkv, Skv, D))).bfloat16().cuda()
    o, lse = attention.gqa_split_fwd(q, k, v, 1.0 / math.sqrt(D), causal=spec["causal"])
    o_np, lse_np = o.float().cpu().numpy(), lse.cpu().numpy()
    res = {}
    ref_o = Path(f"{pre}_o.bin")
    if ref_o.exists():
        res["o_max_abs"] = float(np.abs(o_np - load_bin(ref_o, o_np.shape)).max())
    ref_l = Path(f"{pre}_lse.bin")
    if ref_l.exists():
        res["lse_max_abs"] = float(np.abs(lse_np - load_bin(ref_l, lse_np.shape)).max())
    if write_outputs:
        save_bin(f"{pre}_o_bw.bin", o_np)
        save_bin(f"{pre}_lse_bw.bin", lse_np)
    return res
