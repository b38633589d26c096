"""Golden-file (.bin) interop: round trip of the reference's headerless float32
format, and the C++ helpers compile against the header."""
import subprocess
from pathlib import Path

import numpy as np
import pytest

from blackwell_b200 import binio

ROOT = Path(__file__).resolve().parent.parent


def test_roundtrip(tmp_path):
    a = np.random.default_rng(0).standard_normal((2, 3, 5)).astype(np.float32)
    binio.save_bin(tmp_path / "x.bin", a)
    assert (tmp_path / "x.bin").stat().st_size == a.size * 4
    np.testing.assert_array_equal(binio.load_bin(tmp_path / "x.bin", a.shape), a)
    with pytest.raises(ValueError):
        binio.load_bin(tmp_path / "x.bin", (7,))


def test_cpp_helpers_compile_and_roundtrip(tmp_path):
    src = tmp_path / "t.cpp"
    src.write_text('''
#include "bw_attn_launchers.hpp"
int main(int argc, char** argv) {
  float a[4] = {1.f, -2.5f, 3.25f, 0.f}, b[4] = {};
  if (!bw_compat::saveBin(argv[1], a, 4)) return 1;
  if (!bw_compat::loadBin(argv[1], b, 4)) return 2;
  for (int i = 0; i < 4; ++i) if (a[i] != b[i]) return 3;
  return bw_compat::loadBin(argv[1], b, 5) ? 4 : 0;   // short file must fail
}''')
    exe = tmp_path / "t"
    subprocess.run(["nvcc", "-x", "cu", "-I", str(ROOT / "include"), str(src), "-o", str(exe)], check=True)
    r = subprocess.run([str(exe), str(tmp_path / "v.bin")])
    assert r.returncode == 0
    np.testing.assert_array_equal(binio.load_bin(tmp_path / "v.bin", (4,)), [1, -2.5, 3.25, 0])


@pytest.mark.gpu
def test_run_case_on_reference_format(tmp_path, golden):
    """Write a golden case in the reference's data/ layout and run it."""
    from tests._util import bf16_from_bits
    g = golden("gqa_causal_d128")
    q, k, v = (bf16_from_bits(g[n]).float().numpy() for n in ("q_bf16", "k_bf16", "v_bf16"))
    for name, arr in (("q", q), ("k", k), ("v", v), ("lse", g["lse_fp64"])):
        binio.save_bin(tmp_path / f"gqa_causal_{name}.bin", arr)
    binio.save_bin(tmp_path / "gqa_causal_o.bin", g["o_fp64"])
    B, Hq, S, D = q.shape
    res = binio.run_case(tmp_path, "gqa_causal", B, Hq, k.shape[1], D, S=S)
    assert res["o_max_abs"] <= 2e-2 and res["lse_max_abs"] <= 1e-3
    assert (tmp_path / "gqa_causal_o_bw.bin").exists()
