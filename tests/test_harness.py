"""The C++ host side: CMakeLists.txt builds the library and the reference-style
harness for sm_100a; the harness (bw_harness) reads the reference's data/*.bin
files, runs the launcher templates over the C ABI, checks with the reference's
checkResult rule and benchmarks with its flush-and-events method."""
import ctypes
import re
import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
HARNESS = ROOT / "blackwell_b200" / "bw_harness"


@pytest.mark.skipif(shutil.which("cmake") is None, reason="cmake not installed")
def test_cmake_builds_library_and_harness(tmp_path):
    out = tmp_path / "out"
    subprocess.run(["cmake", "-S", str(ROOT), "-B", str(tmp_path / "b"), f"-DBW_OUTPUT_DIR={out}",
                    "-DCMAKE_CUDA_COMPILER=/usr/local/cuda/bin/nvcc"], check=True, capture_output=True)
    subprocess.run(["cmake", "--build", str(tmp_path / "b"), "-j", "16"], check=True, capture_output=True)
    lib = ctypes.CDLL(str(out / "libbw_attn.so"))
    header = (ROOT / "include" / "bw_attn.h").read_text()
    for sym in sorted(set(re.findall(r"BW_API\s+[\w\s\*]*?\b(bw_\w+)\s*\(", header))):
        assert hasattr(lib, sym), sym
    r = subprocess.run([str(out / "bw_harness")], capture_output=True, text=True)
    assert r.returncode == 2 and "usage" in r.stderr


def test_harness_usage_errors():
    if not HARNESS.exists():
        pytest.skip("harness not built")
    for argv in ([], ["nope"], ["gqa", "--D", "96"], ["gqa", "--B"]):
        assert subprocess.run([str(HARNESS), *argv], capture_output=True).returncode == 2


@pytest.mark.gpu
def test_harness_on_reference_files(tmp_path, golden):
    """A golden case written in the reference's data/ naming: the harness passes
    its checks; a corrupted expected output makes it fail with status 1."""
    from tests._util import bf16_from_bits
    g = golden("gqa_causal_d128")
    q, k, v = (bf16_from_bits(g[n]).float().numpy() for n in ("q_bf16", "k_bf16", "v_bf16"))
    B, Hq, S, D = q.shape
    Hkv = k.shape[1]
    data = tmp_path / "data"
    data.mkdir()
    for name, arr in (("q", q), ("k", k), ("v", v), ("o", g["o_fp64"]), ("lse", g["lse_fp64"])):
        np.asarray(arr, np.float32).tofile(data / f"gqa_causal_{name}.bin")
    args = [str(HARNESS), "gqa_causal", "--B", str(B), "--Hq", str(Hq), "--Hkv", str(Hkv), "--S", str(S),
            "--D", str(D), "--data", str(data), "--iters", "5", "--warmup", "2"]
    r = subprocess.run(args, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.count("Values match!") == 2 and "Median Time" in r.stdout
    bad = np.asarray(g["o_fp64"], np.float32).copy()
    bad.flat[17] += 1.0
    bad.tofile(data / "gqa_causal_o.bin")
    r = subprocess.run(args, capture_output=True, text=True, timeout=300)
    assert r.returncode == 1 and "don't match at index 17" in r.stdout


@pytest.mark.gpu
def test_harness_mha_f32_on_reference_files(tmp_path, golden):
    """fp32 MHA through bw_compat::launch_mha_f32 (the reference's mha_v3_tc call
    shape) on the reference's own fp32 fixture: the harness's check passes at a
    1e-5 tolerance (3xTF32 accuracy); a corrupted expected output fails."""
    g = golden("mha_fp32_d64")
    q, k, v = (np.asarray(g[n], np.float32) for n in ("q_f32", "k_f32", "v_f32"))
    B, H, S, D = q.shape
    data = tmp_path / "data"
    data.mkdir()
    for name, arr in (("q", q), ("k", k), ("v", v), ("out", g["o_fp64"])):
        np.asarray(arr, np.float32).tofile(data / f"mha_{name}.bin")
    args = [str(HARNESS), "mha_f32", "--B", str(B), "--Hq", str(H), "--S", str(S), "--D", "64", "--data", str(data),
            "--iters", "5", "--warmup", "2", "--tol", "1e-5"]
    r = subprocess.run(args, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.count("Values match!") == 1 and "Median Time" in r.stdout
    bad = np.asarray(g["o_fp64"], np.float32).copy()
    bad.flat[5] += 1e-3
    bad.tofile(data / "mha_out.bin")
    r = subprocess.run(args, capture_output=True, text=True, timeout=300)
    assert r.returncode == 1 and "don't match at index 5" in r.stdout
