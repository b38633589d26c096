"""The reference's own split-length GQA kernel (adhitya_GQA.cu launch_gqa_v1,
built unmodified by oracle/build_ref.py) against this library on the same
inputs, at the reference program's fixed shape (B=16, Hq=12, Hkv=4, Sq=4096,
Skv=2048, D=64, non-causal): the reference program reads its expected O and
LSE from data/gqa_split_*.bin, which this test writes from bw.gqa_split_fwd,
and checks them with its own checkResult (atol = rtol = 2e-2).  The timings
of both kernels (the reference's harness: 256 MiB L2 flush, 100 runs; ours:
the same flush, CUDA events) are printed for the record."""
import math
import re
import statistics
import subprocess
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

REF_BIN = Path(__file__).resolve().parent.parent / "oracle" / "_ref" / "adhitya_gqa"


@pytest.mark.skipif(not REF_BIN.exists(), reason="reference program not built (oracle/build_ref.py)")
def test_reference_split_kernel_agrees(tmp_path):
    import blackwell_b200 as bw

    B, Hq, Hkv, Sq, Skv, D = 16, 12, 4, 4096, 2048, 64
    g = torch.Generator().manual_seed(7)
    q = torch.randn(B, Hq, Sq, D, generator=g).bfloat16()
    k = torch.randn(B, Hkv, Skv, D, generator=g).bfloat16()
    v = torch.randn(B, Hkv, Skv, D, generator=g).bfloat16()
    qd, kd, vd = q.cuda(), k.cuda(), v.cuda()
    scale = 1.0 / math.sqrt(D)
    o, lse = bw.gqa_split_fwd(qd, kd, vd, scale)
    assert bw.stream_status() == 0
    data = tmp_path / "data"
    data.mkdir()
    # the reference program reads fp32 .bin files and narrows the inputs to bf16
    for name, t in (("q", q), ("k", k), ("v", v), ("o", o.cpu()), ("lse", lse.cpu())):
        t.float().numpy().astype(np.float32).tofile(data / f"gqa_split_{name}.bin")
    res = subprocess.run([str(REF_BIN)], cwd=tmp_path, capture_output=True, text=True, timeout=600)
    out = res.stdout
    print(out[-1500:])
    assert res.returncode == 0, res.stderr[-2000:]
    assert "Loaded PyTorch reference" in out
    assert out.count("Values match!") == 2, out[-2000:]
    ref_ms = float(re.search(r"Median Time:\s+([\d.]+)", out).group(1))

    # our kernel at the same shape, the same flush, CUDA events
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    times = []
    for i in range(30):
        flush.zero_()
        a, b = torch.cuda.Event(True), torch.cuda.Event(True)
        a.record()
        bw.gqa_split_fwd(qd, kd, vd, scale, out=o, lse=lse)
        b.record()
        torch.cuda.synchronize()
        if i >= 5:
            times.append(a.elapsed_time(b))
    ours = statistics.median(times)
    flops = 4.0 * B * Hq * Sq * Skv * D
    print(f"reference launch_gqa_v1 median {ref_ms:.3f} ms ({flops / ref_ms / 1e9:.1f} TFLOP/s); "
          f"bw_gqa_split_fwd median {ours:.4f} ms ({flops / ours / 1e9:.1f} TFLOP/s); "
          f"speed-up {ref_ms / ours:.1f}x")
    assert ours < ref_ms


REF_GQA = Path(__file__).resolve().parent.parent / "oracle" / "_ref" / "gqa_sm120"


@pytest.mark.skipif(not REF_GQA.exists(), reason="reference program not built (oracle/build_ref.py)")
def test_reference_gqa_kernels_agree(tmp_path):
    """The reference's non-causal GQA kernels (gqa_v1 two-pass, gqa_v2 online
    softmax; GQA_sm120.cu) at their program's shape (B=16, Hq=12, Hkv=4,
    S=4096, D=64) checked by the program's own checkResult against
    bw_gqa_fwd's O and LSE, and timed against it."""
    import blackwell_b200 as bw

    B, Hq, Hkv, S, D = 16, 12, 4, 4096, 64
    g = torch.Generator().manual_seed(13)
    q = torch.randn(B, Hq, S, D, generator=g).bfloat16()
    k = torch.randn(B, Hkv, S, D, generator=g).bfloat16()
    v = torch.randn(B, Hkv, S, D, generator=g).bfloat16()
    qd, kd, vd = q.cuda(), k.cuda(), v.cuda()
    scale = 1.0 / math.sqrt(D)
    o, lse = bw.gqa_fwd(qd, kd, vd, scale)
    assert bw.stream_status() == 0
    data = tmp_path / "data"
    data.mkdir()
    for name, t in (("q", q), ("k", k), ("v", v), ("o", o.cpu()), ("lse", lse.cpu())):
        t.float().numpy().astype(np.float32).tofile(data / f"gqa_{name}.bin")
    res = subprocess.run([str(REF_GQA)], cwd=tmp_path, capture_output=True, text=True, timeout=900)
    out = res.stdout
    print(out[-2500:])
    assert res.returncode == 0, res.stderr[-2000:]
    assert "Loaded PyTorch reference" in out
    assert out.count("Values match!") == 4, out[-2500:]      # O and LSE for V1 and V2
    ref_ms = [float(x) for x in re.findall(r"Median Time:\s+([\d.]+)", out)]
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    times = []
    for i in range(30):
        flush.zero_()
        a, b = torch.cuda.Event(True), torch.cuda.Event(True)
        a.record()
        bw.gqa_fwd(qd, kd, vd, scale, out=o, lse=lse)
        b.record()
        torch.cuda.synchronize()
        if i >= 5:
            times.append(a.elapsed_time(b))
    ours = statistics.median(times)
    flops = 4.0 * B * Hq * S * S * D
    print(f"reference gqa_v1 / gqa_v2 median {ref_ms[0]:.3f} / {ref_ms[1]:.3f} ms "
          f"({flops / ref_ms[0] / 1e9:.1f} / {flops / ref_ms[1] / 1e9:.1f} TFLOP/s); "
          f"bw_gqa_fwd median {ours:.4f} ms ({flops / ours / 1e9:.1f} TFLOP/s); "
          f"speed-up {min(ref_ms) / ours:.1f}x over the faster")
    assert ours < min(ref_ms)


REF_MHA = Path(__file__).resolve().parent.parent / "oracle" / "_ref" / "mha_sm120"


def _max_abs(out, label):
    line = next(ln for ln in out.splitlines() if label in ln)
    return float(re.search(r"max_abs=([\d.eE+-]+)", line).group(1))


@pytest.mark.skipif(not REF_MHA.exists(), reason="reference program not built (oracle/build_ref.py)")
def test_reference_mha_fp32_kernel_agrees(tmp_path):
    """The reference's fp32 MHA kernel (mha_v3_tc, 3xTF32) at its program's
    shape (B=16, H=12, S=1024, D=64) on inputs U[0,1) - 0.5, with the files'
    "SDPA" output = bw_mha_fwd_f32 and their fp64 output = the oracle: the
    reference kernel must sit on the oracle (this pins the oracle with the
    reference's own GPU code), and ours (the same 3xTF32 split on tcgen05
    kind::tf32 MMAs) within 1e-5 of both: fp32 accuracy, like the reference."""
    import blackwell_b200 as bw
    from oracle import attention_oracle as orc

    B, H, S, D = 16, 12, 1024, 64
    g = torch.Generator().manual_seed(11)
    q, k, v = (torch.rand(B, H, S, D, generator=g) - 0.5 for _ in range(3))
    scale = 1.0 / math.sqrt(D)
    o, _ = bw.mha_fwd_f32(q.cuda(), k.cuda(), v.cuda(), scale)
    assert bw.stream_status() == 0
    # fp64 ground truth, batched over heads (same arithmetic as the oracle's
    # per-head restatement of baseline_mha.py:28-33)
    q64, k64, v64 = (t.double() for t in (q, k, v))
    ref64 = torch.softmax(q64 @ k64.transpose(-1, -2) * scale, dim=-1) @ v64
    h0 = orc.fp64_attention(q[:1, :1], k[:1, :1], v[:1, :1], scale)
    assert np.abs(h0 - ref64[:1, :1].numpy()).max() < 1e-6      # same as the oracle
    data = tmp_path / "data"
    data.mkdir()
    for name, t in (("q", q), ("k", k), ("v", v), ("out", o.cpu()), ("out_fp64", ref64)):
        t.float().numpy().astype(np.float32).tofile(data / f"mha_{name}.bin")
    res = subprocess.run([str(REF_MHA)], cwd=tmp_path, capture_output=True, text=True, timeout=600)
    out = res.stdout
    print(out[-1500:])
    assert res.returncode == 0, res.stderr[-2000:]
    ref_vs_fp64 = _max_abs(out, "mha_v3_tc    vs  fp64")
    ours_vs_fp64 = _max_abs(out, "torch.SDPA   vs  fp64")     # the files' "SDPA" slot holds our output
    ref_vs_ours = _max_abs(out, "mha_v3_tc    vs  SDPA")
    assert ref_vs_fp64 <= 1e-5, ref_vs_fp64
    assert ours_vs_fp64 <= 1e-5 and ref_vs_ours <= 1e-5, (ours_vs_fp64, ref_vs_ours)
    ref_ms = float(re.search(r"Median Time:\s+([\d.]+)", out).group(1))
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    qd, kd, vd = q.cuda(), k.cuda(), v.cuda()
    times = []
    for i in range(30):
        flush.zero_()
        a, b = torch.cuda.Event(True), torch.cuda.Event(True)
        a.record()
        bw.mha_fwd_f32(qd, kd, vd, scale)
        b.record()
        torch.cuda.synchronize()
        if i >= 5:
            times.append(a.elapsed_time(b))
    ours = statistics.median(times)
    flops = 4.0 * B * H * S * S * D
    print(f"reference mha_v3_tc median {ref_ms:.3f} ms ({flops / ref_ms / 1e9:.1f} TFLOP/s); "
          f"bw_mha_fwd_f32 median {ours:.4f} ms ({flops / ours / 1e9:.1f} TFLOP/s); speed-up {ref_ms / ours:.1f}x; "
          f"max-abs vs fp64: reference {ref_vs_fp64:.2e}, ours {ours_vs_fp64:.2e}")
    assert ours < ref_ms
