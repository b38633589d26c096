"""The CPU oracle restates the reference's ground truth; pin it to golden vectors
made by the reference's own functions (tests/golden/make_golden.py)."""
import math

import numpy as np
import pytest
import torch

from oracle import attention_oracle as orc
from tests._util import bf16_from_bits

GQA_CASES = ["gqa_nc_d128", "gqa_causal_d128", "gqa_causal_d64_g3_rand", "gqa_causal_d64_ragged", "gqa_split_d64"]


def _inputs(g):
    if "q_bf16" in g:
        return [bf16_from_bits(g[k]).float() for k in ("q_bf16", "k_bf16", "v_bf16")]
    return [torch.from_numpy(g[k]) for k in ("q_f32", "k_f32", "v_f32")]


@pytest.mark.parametrize("name", GQA_CASES + ["c1_gqa_fp32"])
def test_oracle_matches_reference_golden(golden, name):
    g = golden(name)
    q, k, v = _inputs(g)
    o, lse = orc.fp64_reference(q, k, v, float(g["scale"]), causal=bool(g["causal"]))
    np.testing.assert_allclose(o, g["o_fp64"], atol=2e-6, rtol=0)
    np.testing.assert_allclose(lse, g["lse_fp64"], atol=2e-6, rtol=0)


def test_c1_cpu_sdpa_path_matches_fp64(golden):
    """C1 (CPU plumbing): the reference's CPU execution path (torch SDPA, fp32)
    against its fp64 ground truth, and against the SDPA output it produced."""
    g = golden("c1_gqa_fp32")
    q, k, v = _inputs(g)
    o = orc.sdpa_cpu(q, k, v, float(g["scale"]))
    assert np.abs(o.numpy() - g["o_fp64"]).max() < 1e-5
    assert np.abs(o.numpy() - g["o_sdpa"]).max() < 1e-5


def test_mha_oracle(golden):
    g = golden("mha_fp32_d64")
    q, k, v = _inputs(g)
    o = orc.fp64_attention(q, k, v, float(g["scale"]))
    np.testing.assert_allclose(o, g["o_fp64"], atol=2e-6, rtol=0)


def test_decode_oracle(golden):
    g = golden("decode_d128")
    q, k, v = (bf16_from_bits(g[n]).float() for n in ("q_bf16", "k_bf16", "v_bf16"))
    o, lse = orc.decode_reference(q, k, v, g["kv_lens"], g["kv_offsets"], float(g["scale"]))
    np.testing.assert_allclose(o, g["o_fp64"], atol=2e-6, rtol=0)
    np.testing.assert_allclose(lse, g["lse_fp64"], atol=2e-6, rtol=0)


def test_rows_oracle_equals_full(golden):
    g = golden("gqa_causal_d64_g3_rand")
    q, k, v = _inputs(g)
    rng = np.random.default_rng(0)
    B, Hq, S, _ = q.shape
    rows = np.stack([rng.integers(0, B, 20), rng.integers(0, Hq, 20), rng.integers(0, S, 20)], 1)
    o, lse = orc.fp64_rows(q, k, v, float(g["scale"]), True, rows)
    for r, (b, h, i) in enumerate(rows):
        assert np.abs(o[r] - g["o_fp64"][b, h, i]).max() < 2e-6
        assert abs(lse[r] - g["lse_fp64"][b, h, i]) < 2e-6


@pytest.mark.parametrize("splits", [1, 2, 5, 64])
def test_lse_combine_identity(splits):
    """combine(partials of a split) == unsplit result (the merge identity)."""
    rng = np.random.default_rng(splits)
    L, D = 640, 64
    q = rng.standard_normal((1, 1, 1, D))
    k = rng.standard_normal((1, 1, L, D))
    v = rng.standard_normal((1, 1, L, D))
    scale = 1 / math.sqrt(D)
    full_o, full_l = orc.fp64_reference(q, k, v, scale)
    bounds = np.linspace(0, L, splits + 1).astype(int)
    ops, lps = [], []
    for s in range(splits):
        a, b = bounds[s], bounds[s + 1]
        o, l = orc.fp64_reference(q, k[:, :, a:b], v[:, :, a:b], scale)
        ops.append(o[0, 0])
        lps.append(l[0, 0])
    o, l = orc.lse_combine_reference(np.stack(ops), np.stack(lps))
    np.testing.assert_allclose(o, full_o[0, 0], atol=1e-6)
    np.testing.assert_allclose(l, full_l[0, 0], atol=1e-6)


def test_lse_combine_empty_split():
    o = np.zeros((2, 3, 8))
    o[0] = 1.0
    l = np.array([[0.5, 0.1, 2.0], [-np.inf] * 3])
    out, lse = orc.lse_combine_reference(o, l)
    np.testing.assert_allclose(out, 1.0)
    np.testing.assert_allclose(lse, l[0], rtol=1e-6)


def test_fp64_rows_query_offset_matches_full_causal():
    """fp64_rows with q_offset (query i at sequence position q_offset + i) gives
    the tail rows of the top-left-aligned causal reference on the full sequence."""
    rng = np.random.default_rng(5)
    B, Hq, Hkv, S, D, off = 1, 2, 1, 40, 16, 25
    q = rng.standard_normal((B, Hq, S, D))
    k = rng.standard_normal((B, Hkv, S, D))
    v = rng.standard_normal((B, Hkv, S, D))
    full_o, full_l = orc.fp64_reference(q, k, v, 0.25, causal=True)
    rows = np.array([[0, h, i] for h in range(Hq) for i in range(S - off)])
    o, l = orc.fp64_rows(q[:, :, off:], k, v, 0.25, True, rows, q_offset=off)
    np.testing.assert_allclose(o, full_o[0, :, off:].reshape(-1, D), rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(l, full_l[0, :, off:].reshape(-1), rtol=1e-6, atol=1e-6)
