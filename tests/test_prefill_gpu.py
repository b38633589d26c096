"""Parity of the sm_100a attention forward (through the C ABI) with the oracle.

Bar: max-abs error <= 2e-2 on bf16 O and <= 1e-3 on LSE against the fp64
restatement of the reference's ground truth, on the same bf16 input bits."""
import math

import numpy as np
import pytest
import torch

from oracle import attention_oracle as orc
from tests._util import LSE_TOL, O_TOL, bf16_from_bits, seeded_bf16

pytestmark = pytest.mark.gpu

GOLDEN_GQA = ["gqa_nc_d128", "gqa_causal_d128", "gqa_causal_d64_g3_rand", "gqa_causal_d64_ragged", "gqa_split_d64"]


@pytest.fixture(scope="module", params=[0, 4], ids=["default", "k4_one_acc"])
def p_variant(request):
    """Prefill kernels: the default (kernel 5 at D = 64: alternate key tiles per
    softmax warpgroup into two accumulators; kernel 4 at D = 128) and kernel 4
    at both head dimensions (three score buffers, one accumulator, four threads
    per row)."""
    import blackwell_b200 as bw
    from blackwell_b200 import _ffi
    old = bw.get_option(_ffi.BW_OPT_PREFILL_KERNEL)
    bw.set_option(_ffi.BW_OPT_PREFILL_KERNEL, request.param)
    yield request.param
    bw.set_option(_ffi.BW_OPT_PREFILL_KERNEL, old)


def _run(q, k, v, scale, causal):
    import blackwell_b200 as bw
    o, lse = bw.gqa_split_fwd(q.cuda(), k.cuda(), v.cuda(), scale, causal=causal)
    assert bw.stream_status() == 0
    return o.float().cpu().numpy(), lse.cpu().numpy()


@pytest.mark.parametrize("name", GOLDEN_GQA)
def test_golden(golden, name, p_variant):
    g = golden(name)
    q, k, v = (bf16_from_bits(g[n]) for n in ("q_bf16", "k_bf16", "v_bf16"))
    o, lse = _run(q, k, v, float(g["scale"]), bool(g["causal"]))
    assert np.abs(o - g["o_fp64"]).max() <= O_TOL
    assert np.abs(lse - g["lse_fp64"]).max() <= LSE_TOL


def test_c1_shape_in_bf16(golden, p_variant):
    """C1's shape (B=1,Hq=8,Hkv=2,S=512,D=64) on the GPU, inputs rounded to bf16."""
    g = golden("c1_gqa_fp32")
    q, k, v = (torch.from_numpy(g[n]).bfloat16() for n in ("q_f32", "k_f32", "v_f32"))
    o, lse = _run(q, k, v, float(g["scale"]), False)
    ro, rl = orc.fp64_reference(q.float(), k.float(), v.float(), float(g["scale"]))
    assert np.abs(o - ro).max() <= O_TOL
    assert np.abs(lse - rl).max() <= LSE_TOL


CASES = [
    # B, Hq, Hkv, Sq, Skv, D, causal
    (1, 2, 2, 1, 1, 64, False),
    (1, 2, 1, 1, 1, 128, True),
    (2, 4, 4, 77, 77, 64, True),      # MHA, ragged S
    (1, 8, 1, 128, 128, 128, True),    # G = 8
    (1, 3, 1, 300, 300, 128, False),   # G = 3 (odd: query-tile pairs)
    (2, 4, 2, 513, 513, 128, True),
    (1, 6, 2, 257, 640, 64, False),    # split lengths
    (1, 4, 2, 640, 200, 128, True),    # Sq > Skv, causal
    (1, 2, 1, 1, 1000, 128, False),    # one query row
    (2, 6, 2, 640, 640, 64, True),     # odd key-tile counts per causal segment (5 + 1, 3 + 3)
    (1, 4, 1, 1000, 1000, 64, True),   # 8 query tiles: segments of 8 + 1 .. 5 + 4 key tiles
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "x".join(map(str, c)))
def test_shapes(case, p_variant):
    B, Hq, Hkv, Sq, Skv, D, causal = case
    q = seeded_bf16((B, Hq, Sq, D), 1)
    k = seeded_bf16((B, Hkv, Skv, D), 2)
    v = seeded_bf16((B, Hkv, Skv, D), 3)
    scale = 1 / math.sqrt(D)
    o, lse = _run(q, k, v, scale, causal)
    ro, rl = orc.fp64_reference(q.float(), k.float(), v.float(), scale, causal=causal)
    assert np.abs(o - ro).max() <= O_TOL
    assert np.abs(lse - rl).max() <= LSE_TOL
    # tighter statistical check: bf16 rounding of O alone gives a mean error of a
    # few 1e-4; systematic softmax errors (a wrong max, a wrong mask) show up here
    assert np.abs(o - ro).mean() <= 2e-3
    if causal:
        # query row 0 sees only key 0, so O[row 0] is exactly V[0]
        G = Hq // Hkv
        np.testing.assert_array_equal(o[:, :, 0], v[:, :, 0].float().numpy().repeat(G, axis=1))


def test_bshd_layout_strides():
    """BSHD storage passed through strides (the C2 layout), no copies."""
    import blackwell_b200 as bw
    B, S, Hq, Hkv, D = 2, 384, 8, 2, 128
    qs = seeded_bf16((B, S, Hq, D), 4)
    ks = seeded_bf16((B, S, Hkv, D), 5)
    vs = seeded_bf16((B, S, Hkv, D), 6)
    out = torch.empty((B, S, Hq, D), dtype=torch.bfloat16, device="cuda")
    o, lse = bw.gqa_causal_fwd(qs.cuda().transpose(1, 2), ks.cuda().transpose(1, 2), vs.cuda().transpose(1, 2),
                               1 / math.sqrt(D), out=out.transpose(1, 2))
    assert bw.stream_status() == 0
    ro, rl = orc.fp64_reference(qs.transpose(1, 2).float(), ks.transpose(1, 2).float(), vs.transpose(1, 2).float(),
                                1 / math.sqrt(D), causal=True)
    assert np.abs(out.transpose(1, 2).float().cpu().numpy() - ro).max() <= O_TOL
    assert np.abs(lse.cpu().numpy() - rl).max() <= LSE_TOL


def test_c2_full_size_rows():
    """C2 at full size (B=4,Hq=32,Hkv=8,S=4096,D=128, causal, BSHD): 2048 random
    rows against the fp64 row oracle, plus size-independent properties."""
    import blackwell_b200 as bw
    B, S, Hq, Hkv, D = 4, 4096, 32, 8, 128
    g = torch.Generator(device="cuda").manual_seed(42)
    q = torch.randn(B, S, Hq, D, generator=g, device="cuda").bfloat16()
    k = torch.randn(B, S, Hkv, D, generator=g, device="cuda").bfloat16()
    v = torch.randn(B, S, Hkv, D, generator=g, device="cuda").bfloat16()
    qt, kt, vt = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
    o, lse = bw.gqa_causal_fwd(qt, kt, vt, 1 / math.sqrt(D))
    assert bw.stream_status() == 0
    assert torch.isfinite(o.float()).all() and torch.isfinite(lse).all()
    rng = np.random.default_rng(7)
    rows = np.stack([rng.integers(0, B, 2048), rng.integers(0, Hq, 2048), rng.integers(0, S, 2048)], 1)
    rows[:8, 2] = [0, 1, 127, 128, 4095, 4094, 2047, 2048]
    qc, kc, vc = qt.float().cpu(), kt.float().cpu(), vt.float().cpu()
    ro, rl = orc.fp64_rows(qc, kc, vc, 1 / math.sqrt(D), True, rows)
    oc, lc = o.float().cpu().numpy(), lse.cpu().numpy()
    got_o = np.stack([oc[b, h, i] for b, h, i in rows])
    got_l = np.array([lc[b, h, i] for b, h, i in rows])
    assert np.abs(got_o - ro).max() <= O_TOL
    assert np.abs(got_l - rl).max() <= LSE_TOL
    # row 0 sees only key 0: O = V[0]
    assert torch.allclose(o[:, :, 0].float(), vt[:, :, 0].repeat_interleave(Hq // Hkv, 1).float(), atol=1e-2)


def test_deterministic_and_out_of_place():
    import blackwell_b200 as bw
    q = seeded_bf16((1, 4, 700, 128), 8).cuda()
    k = seeded_bf16((1, 2, 700, 128), 9).cuda()
    v = seeded_bf16((1, 2, 700, 128), 10).cuda()
    o1, l1 = bw.gqa_causal_fwd(q, k, v)
    o2, l2 = bw.gqa_causal_fwd(q, k, v)
    assert torch.equal(o1, o2) and torch.equal(l1, l2)


@pytest.mark.parametrize("poly", [0, 2, 3, 4])
@pytest.mark.parametrize("name", ["gqa_causal_d128", "gqa_causal_d64_g3_rand"])
def test_exp_poly_split(golden, name, poly):
    """Every supported MUFU / polynomial split of the softmax exponentials meets the bar."""
    import blackwell_b200 as bw
    from blackwell_b200 import _ffi
    old = bw.get_option(_ffi.BW_OPT_EXP_POLY)
    bw.set_option(_ffi.BW_OPT_EXP_POLY, poly)
    try:
        g = golden(name)
        q, k, v = (bf16_from_bits(g[n]) for n in ("q_bf16", "k_bf16", "v_bf16"))
        o, lse = _run(q, k, v, float(g["scale"]), bool(g["causal"]))
    finally:
        bw.set_option(_ffi.BW_OPT_EXP_POLY, old)
    assert np.abs(o - g["o_fp64"]).max() <= O_TOL
    assert np.abs(o - g["o_fp64"]).mean() <= 2e-3
    assert np.abs(lse - g["lse_fp64"]).max() <= LSE_TOL


def test_long_context_rows():
    """C5's per-GPU slice shape (one KV group: Hq=8 query heads, Hkv=1, D=128,
    causal) at S = 65536: 160 rows (including the first and last tiles) against
    the fp64 row oracle."""
    import blackwell_b200 as bw
    B, Hq, Hkv, S, D = 1, 8, 1, 65536, 128
    g = torch.Generator(device="cuda").manual_seed(5)
    q = torch.randn(B, Hq, S, D, generator=g, device="cuda").bfloat16()
    k = torch.randn(B, Hkv, S, D, generator=g, device="cuda").bfloat16()
    v = torch.randn(B, Hkv, S, D, generator=g, device="cuda").bfloat16()
    o, lse = bw.gqa_causal_fwd(q, k, v)
    assert bw.stream_status() == 0
    rng = np.random.default_rng(11)
    rows = np.stack([np.zeros(160, int), rng.integers(0, Hq, 160), rng.integers(0, S, 160)], 1)
    rows[:6, 2] = [0, 127, 128, S - 129, S - 128, S - 1]
    qc, kc, vc = q.float().cpu(), k.float().cpu(), v.float().cpu()
    ro, rl = orc.fp64_rows(qc, kc, vc, 1 / math.sqrt(D), True, rows)
    oc, lc = o.float().cpu().numpy(), lse.cpu().numpy()
    assert np.abs(np.stack([oc[b, h, i] for b, h, i in rows]) - ro).max() <= O_TOL
    assert np.abs(np.array([lc[b, h, i] for b, h, i in rows]) - rl).max() <= LSE_TOL


@pytest.mark.parametrize("layout,causal,S,chunks,D", [
    ("bshd", True, 320, 1, 128), ("bshd", True, 320, 3, 128), ("bshd", True, 1000, 8, 128),
    ("bhsd", True, 777, 4, 128), ("bshd", False, 320, 3, 128), ("bhsd", False, 200, 2, 128),
    ("bhsd", True, 64, 4, 128), ("bshd", True, 1000, 5, 64), ("bhsd", True, 513, 3, 64),
])
def test_attention_from_host_pipelined(layout, causal, S, chunks, D):
    """bw_attn_fwd_host (copy-in / kernel / copy-out pipelined in sequence or
    batch chunks; causal chunks run with a query offset) gives the same bits as
    the device path."""
    import blackwell_b200 as bw
    B, Hq, Hkv = 3, 8, 2
    shp = (lambda h: (B, S, h, D)) if layout == "bshd" else (lambda h: (B, h, S, D))
    view = (lambda t: t.transpose(1, 2)) if layout == "bshd" else (lambda t: t)
    q = seeded_bf16(shp(Hq), 61).pin_memory()
    k = seeded_bf16(shp(Hkv), 62).pin_memory()
    v = seeded_bf16(shp(Hkv), 63).pin_memory()
    o = torch.empty(shp(Hq), dtype=torch.bfloat16).pin_memory()
    lse = torch.empty(B, Hq, S, dtype=torch.float32).pin_memory()
    bw.attention_from_host(view(q), view(k), view(v), view(o), lse, causal=causal, chunks=chunks)
    torch.cuda.synchronize()
    assert bw.stream_status() == 0
    fn = bw.gqa_causal_fwd if causal else bw.gqa_fwd
    ro, rl = fn(view(q.cuda()), view(k.cuda()), view(v.cuda()))
    assert torch.equal(view(o), ro.cpu()) and torch.equal(lse, rl.cpu())


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("q_offset,Sq,Skv", [(0, 200, 200), (1, 130, 131), (77, 300, 377), (128, 256, 384),
                                               (300, 129, 1000), (1000, 64, 1064)])
def test_causal_offset(D, q_offset, Sq, Skv):
    """Chunked-prefill causal mask (query i sees keys j <= q_offset + i) against
    the fp64 oracle on every row, and equal to the matching rows of a full causal
    call when the chunk is the sequence tail."""
    import blackwell_b200 as bw
    B, Hq, Hkv = 2, 4, 2
    q = seeded_bf16((B, Hq, Sq, D), 71)
    k, v = seeded_bf16((B, Hkv, Skv, D), 72), seeded_bf16((B, Hkv, Skv, D), 73)
    o, lse = bw.gqa_causal_offset_fwd(q.cuda(), k.cuda(), v.cuda(), q_offset)
    assert bw.stream_status() == 0
    rows = np.array([[b, h, i] for b in range(B) for h in range(Hq) for i in range(Sq)])
    ro, rl = orc.fp64_rows(q, k, v, 1 / math.sqrt(D), True, rows, q_offset=q_offset)
    oc, lc = o.float().cpu().numpy().reshape(-1, D), lse.cpu().numpy().reshape(-1)
    assert np.abs(oc - ro).max() <= O_TOL
    assert np.abs(lc - rl).max() <= LSE_TOL
    if q_offset + Sq == Skv:
        qf = torch.cat([seeded_bf16((B, Hq, q_offset, D), 74), q], dim=2) if q_offset else q
        fo, fl = bw.gqa_causal_fwd(qf.cuda(), k.cuda(), v.cuda())
        assert (fo[:, :, q_offset:].float() - o.float()).abs().max().item() <= 2 ** -7
        assert (fl[:, :, q_offset:] - lse).abs().max().item() <= 1e-4


def test_mha_fp32_golden(golden):
    """fp32 MHA (the reference's mha_v3_tc data types and its 3xTF32 split)
    against the reference's fp64 ground truth on its own input distribution
    (U[0,1) - 0.5, fp32): fp32 accuracy, <= 1e-5."""
    import blackwell_b200 as bw
    g = golden("mha_fp32_d64")
    q, k, v = (torch.from_numpy(g[n]).cuda() for n in ("q_f32", "k_f32", "v_f32"))
    o, lse = bw.mha_fwd_f32(q, k, v, float(g["scale"]))
    assert bw.stream_status() == 0
    err = np.abs(o.cpu().numpy() - g["o_fp64"]).max()
    assert err <= 1e-5, err


@pytest.mark.parametrize("S", [1, 31, 33, 100, 384, 1000])
def test_mha_fp32_shapes(S):
    """Ragged lengths (partial 32-key stages and 128-row query tiles), N(0,1)
    inputs, O and LSE at fp32 accuracy against the fp64 oracle."""
    import blackwell_b200 as bw
    B, H, D = 2, 3, 64
    g = torch.Generator().manual_seed(S)
    q, k, v = (torch.randn(B, H, S, D, generator=g) for _ in range(3))
    o, lse = bw.mha_fwd_f32(q.cuda(), k.cuda(), v.cuda())
    assert bw.stream_status() == 0
    ro, rl = orc.fp64_reference(q, k, v, 1 / math.sqrt(D))
    assert np.abs(o.cpu().numpy() - ro).max() <= 1e-5
    assert np.abs(lse.cpu().numpy() - rl).max() <= 1e-5


def test_mha_fp32_strided_out_and_reuse():
    """BSHD strides for inputs and output, and two calls in a row on one workspace."""
    import blackwell_b200 as bw
    B, S, H, D = 2, 300, 4, 64
    g = torch.Generator().manual_seed(5)
    q, k, v = (torch.randn(B, S, H, D, generator=g) for _ in range(3))
    out = torch.empty(B, S, H, D, device="cuda")
    for _ in range(2):
        o, lse = bw.mha_fwd_f32(q.cuda().transpose(1, 2), k.cuda().transpose(1, 2), v.cuda().transpose(1, 2),
                                out=out.transpose(1, 2))
        assert bw.stream_status() == 0
        ro, rl = orc.fp64_reference(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), 1 / math.sqrt(D))
        assert np.abs(out.transpose(1, 2).cpu().numpy() - ro).max() <= 1e-5


@pytest.mark.parametrize("kernel,D", [(4, 128), (5, 64), (4, 64)])
@pytest.mark.parametrize("q_scale,causal", [(12.0, True), (12.0, False), (0.02, True)])
def test_logit_range_stress(kernel, D, q_scale, causal):
    """Large logits (q scaled up: the running max moves by far more than the
    lazy-rescale threshold, and the two parts of a row in kernel 5 end with
    very different maxima) and nearly flat ones, against fp64 rows."""
    import blackwell_b200 as bw
    from blackwell_b200 import _ffi
    B, Hq, Hkv, S = 1, 4, 2, 640
    g = torch.Generator().manual_seed(int(q_scale * 10) + causal)
    # keys with a growing trend so that later tiles keep raising the row max
    q = (torch.randn(B, Hq, S, D, generator=g) * q_scale / math.sqrt(D)).bfloat16()
    k = (torch.randn(B, Hkv, S, D, generator=g) + torch.linspace(0, 3, S)[None, None, :, None]).bfloat16()
    v = torch.randn(B, Hkv, S, D, generator=g).bfloat16()
    old = bw.get_option(_ffi.BW_OPT_PREFILL_KERNEL)
    try:
        bw.set_option(_ffi.BW_OPT_PREFILL_KERNEL, kernel)
        o, lse = bw.gqa_split_fwd(q.cuda(), k.cuda(), v.cuda(), 1 / math.sqrt(D), causal=causal)
        assert bw.stream_status() == 0
    finally:
        bw.set_option(_ffi.BW_OPT_PREFILL_KERNEL, old)
    rows = np.array([[0, h, i] for h in range(Hq) for i in range(0, S, 7)])
    ro, rl = orc.fp64_rows(q, k, v, 1 / math.sqrt(D), causal, rows)
    oc = o.float().cpu().numpy()[0][rows[:, 1], rows[:, 2]]
    lc = lse.cpu().numpy()[0][rows[:, 1], rows[:, 2]]
    assert np.isfinite(oc).all() and np.isfinite(lc).all()
    assert np.abs(oc - ro).max() <= O_TOL
    assert np.abs(lc - rl).max() <= LSE_TOL
