"""The QK-norm + RoPE prologue and the fused op, pinned by the reference's own
ground truth.

The reference checks its fused kernel against two naive GPU kernels of its own,
ref_norm_rope and ref_attention (src/SM103/attention/GQA_fused_sm103.cu:328-420).
oracle/build_ref.py builds them, unmodified, into oracle/_ref/ref_fused (driver:
oracle/ref_fused_driver.cu); this test runs that program on the test's inputs
and compares, on the same bits:

* the oracle's restatement (oracle.norm_rope_reference) with the reference's
  normalised + rotated Q and K: equal but for a rare flip of one bf16 step (the
  two sum the squares in a different order) -- this pins the restatement;
* bw_qk_norm_rope with the reference's Qn / Kn (same rule) and rstd (fp32);
* bw_gqa_fused_fwd's O and LSE with the reference's O and LSE: the reference
  rounds P to bf16 like the kernel; bar O <= 2e-2, LSE <= 1e-3;
* the fp64 attention of the reference's own Qn / Kn with the reference's O
  (the checker agrees with itself)."""
import math
import subprocess
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import attention_oracle as orc
from tests._util import LSE_TOL, O_TOL, seeded_bf16

pytestmark = pytest.mark.gpu

REF_BIN = Path(__file__).resolve().parent.parent / "oracle" / "_ref" / "ref_fused"


def _bf16_bits(t):
    return t.contiguous().view(torch.int16).numpy().astype(np.uint16)


def _rows_agree(a_bits, b_bits):
    """Fraction of bf16 elements that differ, and the largest difference relative
    to the largest magnitude of its row.  A 1-ulp flip of the normalised value
    (the two sides sum the squares in a different order) can turn into a 2-ulp
    step of a small rotated output, so the second figure, not an ulp count, is
    the bound: one bf16 step of the row's scale is 2^-7."""
    f = lambda bits: torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16).float().numpy()
    a, b = f(a_bits), f(b_bits)
    scale = np.maximum(np.abs(b).max(axis=-1, keepdims=True), 1e-30)
    return float((a != b).mean()), float((np.abs(a - b) / scale).max())


@pytest.mark.skipif(not REF_BIN.exists(), reason="reference program not built (oracle/build_ref.py)")
@pytest.mark.parametrize("D,Hq,Hkv,S,neox,causal,use_norm,pos_offset,cache_len", [
    (128, 8, 2, 300, True, True, True, 0, 300),
    (64, 6, 2, 257, False, False, True, 5, 400),
    (128, 4, 4, 200, True, False, False, 3, 150),     # RoPE only, partly beyond the cache
    (64, 12, 4, 512, True, True, True, 0, 512),       # the reference program's head layout (G=3)
])
def test_fused_op_against_reference_ground_truth(tmp_path, D, Hq, Hkv, S, neox, causal, use_norm, pos_offset,
                                                 cache_len):
    import blackwell_b200 as bw
    B, eps = 2, 1e-6
    q, k, v = seeded_bf16((B, Hq, S, D), 81), seeded_bf16((B, Hkv, S, D), 82), seeded_bf16((B, Hkv, S, D), 83)
    cache = orc.rope_cache(cache_len, D)
    g = torch.Generator().manual_seed(9)
    qg = (0.5 + torch.rand(D, generator=g)).float()    # the reference's U[0.5, 1.5) gamma
    kg = (0.5 + torch.rand(D, generator=g)).float()
    for name, t in (("q", q), ("k", k), ("v", v)):
        _bf16_bits(t).tofile(tmp_path / f"{name}.bin")
    cache.astype(np.float32).tofile(tmp_path / "cache.bin")
    qg.numpy().tofile(tmp_path / "qg.bin")
    kg.numpy().tofile(tmp_path / "kg.bin")
    args = [str(REF_BIN), str(tmp_path), B, Hq, Hkv, S, D, int(neox), int(causal), int(use_norm), pos_offset,
            cache_len, eps]
    res = subprocess.run([str(a) for a in args], capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stderr[-2000:]
    rd = lambda n, dt, shape: np.fromfile(tmp_path / f"{n}.bin", dtype=dt).reshape(shape)
    ref_qn = rd("qn", np.uint16, (B, Hq, S, D))
    ref_kn = rd("kn", np.uint16, (B, Hkv, S, D))
    ref_o = torch.from_numpy(rd("o", np.uint16, (B, Hq, S, D)).view(np.int16).copy()).view(torch.bfloat16).float()
    ref_lse = rd("lse", np.float32, (B, Hq, S))

    # 1. the oracle's restatement against the reference's ground truth
    gam = (qg.numpy(), kg.numpy()) if use_norm else (None, None)
    oq, orq = orc.norm_rope_reference(q.float().numpy(), cache, gam[0], eps, pos_offset, not neox)
    ok_, ork = orc.norm_rope_reference(k.float().numpy(), cache, gam[1], eps, pos_offset, not neox)
    for mine, ref in ((oq, ref_qn), (ok_, ref_kn)):
        frac, rel = _rows_agree(_bf16_bits(torch.from_numpy(mine).bfloat16()), ref)
        assert frac <= 2e-3 and rel <= 2 ** -7, (frac, rel)

    # 2. the library's prologue kernel
    cu = lambda t: t.cuda() if t is not None else None
    cache_d = torch.from_numpy(cache).cuda()
    qgd, kgd = (cu(qg), cu(kg)) if use_norm else (None, None)
    q2 = bw.qk_norm_rope(q.cuda(), cache_d, qgd, eps=eps, pos_offset=pos_offset, interleaved=not neox)
    k2 = bw.qk_norm_rope(k.cuda(), cache_d, kgd, eps=eps, pos_offset=pos_offset, interleaved=not neox)
    assert bw.stream_status() == 0
    for mine, ref in ((q2, ref_qn), (k2, ref_kn)):
        frac, rel = _rows_agree(_bf16_bits(mine.cpu()), ref)
        assert frac <= 2e-3 and rel <= 2 ** -7, (frac, rel)

    # 3. the fused entry point against the reference's O and LSE
    o, lse, qr, kr = bw.gqa_fused_fwd(q.cuda(), k.cuda(), v.cuda(), cache_d, qgd, kgd, eps=eps, pos_offset=pos_offset,
                                      interleaved=not neox, causal=causal)
    assert bw.stream_status() == 0
    assert (o.float().cpu() - ref_o).abs().max().item() <= O_TOL
    assert np.abs(lse.cpu().numpy() - ref_lse).max() <= LSE_TOL
    if use_norm:
        np.testing.assert_allclose(qr.cpu().numpy(), rd("qrstd", np.float32, (B, Hq, S)), rtol=1e-5)
        np.testing.assert_allclose(kr.cpu().numpy(), rd("krstd", np.float32, (B, Hkv, S)), rtol=1e-5)

    # 4. the fp64 oracle on the reference's own normalised inputs
    tq = torch.from_numpy(ref_qn.view(np.int16).copy()).view(torch.bfloat16).float()
    tk = torch.from_numpy(ref_kn.view(np.int16).copy()).view(torch.bfloat16).float()
    fo, fl = orc.fp64_reference(tq, tk, v.float(), 1 / math.sqrt(D), causal=causal)
    assert (torch.from_numpy(fo) - ref_o).abs().max().item() <= O_TOL
    assert np.abs(fl - ref_lse).max() <= LSE_TOL
