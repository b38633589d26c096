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
