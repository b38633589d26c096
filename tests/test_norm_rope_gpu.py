"""QK-norm + RoPE prologue and the fused attention op against the restated
reference math (GQA_fused_sm103.cu:59-104): same bf16 rounding points, so the
prologue matches to one bf16 step (fp32 summation order differs)."""
import math

import numpy as np
import pytest
import torch

from oracle import attention_oracle as orc
from tests._util import LSE_TOL, O_TOL, seeded_bf16

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("interleaved", [False, True])
@pytest.mark.parametrize("with_norm", [True, False])
def test_norm_rope(D, interleaved, with_norm):
    import blackwell_b200 as bw
    B, H, S = 2, 3, 150
    x = seeded_bf16((B, H, S, D), 41)
    cache = orc.rope_cache(140, D)           # positions >= 140 stay unrotated
    gamma = (1 + 0.1 * torch.randn(D, generator=torch.Generator().manual_seed(2))).float() if with_norm else None
    y, rstd = bw.qk_norm_rope(x.cuda(), torch.from_numpy(cache).cuda(), gamma.cuda() if with_norm else None,
                              eps=1e-6, pos_offset=-3, interleaved=interleaved, return_rstd=True)
    assert bw.stream_status() == 0
    ry, rr = orc.norm_rope_reference(x.float().numpy(), cache, gamma.numpy() if with_norm else None, 1e-6, -3,
                                     interleaved)
    got = y.float().cpu().numpy()
    # A one-step difference of the normalised inputs (fp32 summation order) moves a
    # rotated output by at most about one bf16 step of the row's largest entries
    # (cancellation in a*c - b*s makes a relative bound on the output too tight).
    row_max = np.abs(ry).max(-1, keepdims=True)
    assert np.all(np.abs(got - ry) <= (np.abs(ry) + row_max) * 2 ** -7 + 1e-6)
    assert np.mean(got == ry) > 0.99
    if with_norm:
        np.testing.assert_allclose(rstd.cpu().numpy(), rr, rtol=1e-5)


@pytest.mark.parametrize("D,Hq,Hkv,S,interleaved,with_norm,causal,pos_offset,cache_len", [
    (128, 4, 2, 300, False, True, True, 0, 300),      # G even: two heads per work item
    (128, 6, 2, 333, True, True, False, 5, 200),      # G odd: two query tiles per item; partly unrotated
    (64, 8, 1, 257, False, False, True, -7, 400),     # RoPE only, negative offset
    (64, 3, 3, 129, True, True, True, 0, 129),        # MHA
])
def test_fused_attention(D, Hq, Hkv, S, interleaved, with_norm, causal, pos_offset, cache_len):
    """The fused op (bw_gqa_fused_fwd: the Q and K prologues as streaming passes
    into the workspace, then the attention kernel) against the restated
    reference math, and bit-identical to composing the public pieces by hand."""
    import blackwell_b200 as bw
    B = 2
    q, k, v = seeded_bf16((B, Hq, S, D), 51), seeded_bf16((B, Hkv, S, D), 52), seeded_bf16((B, Hkv, S, D), 53)
    cache = orc.rope_cache(cache_len, D)
    g = torch.Generator().manual_seed(3)
    qg = (1 + 0.1 * torch.randn(D, generator=g)).float() if with_norm else None
    kg = (1 + 0.1 * torch.randn(D, generator=g)).float() if with_norm else None
    cu = lambda t: t.cuda() if t is not None else None
    o, lse, qr, kr = bw.gqa_fused_fwd(q.cuda(), k.cuda(), v.cuda(), torch.from_numpy(cache).cuda(), cu(qg), cu(kg),
                                      pos_offset=pos_offset, interleaved=interleaved, causal=causal)
    assert bw.stream_status() == 0
    npg = lambda t: t.numpy() if t is not None else None
    q2, rq = orc.norm_rope_reference(q.float().numpy(), cache, npg(qg), 1e-6, pos_offset, interleaved)
    k2, rk = orc.norm_rope_reference(k.float().numpy(), cache, npg(kg), 1e-6, pos_offset, interleaved)
    ro, rl = orc.fp64_reference(q2, k2, v.float(), 1 / math.sqrt(D), causal=causal)
    assert np.abs(o.float().cpu().numpy() - ro).max() <= O_TOL
    assert np.abs(lse.cpu().numpy() - rl).max() <= LSE_TOL
    if with_norm:
        np.testing.assert_allclose(qr.cpu().numpy(), rq, rtol=1e-5)
        np.testing.assert_allclose(kr.cpu().numpy(), rk, rtol=1e-5)
    # composing bw_qk_norm_rope + the attention entry by hand gives the same bits
    q3 = bw.qk_norm_rope(q.cuda(), torch.from_numpy(cache).cuda(), cu(qg), pos_offset=pos_offset,
                         interleaved=interleaved)
    k3 = bw.qk_norm_rope(k.cuda(), torch.from_numpy(cache).cuda(), cu(kg), pos_offset=pos_offset,
                         interleaved=interleaved)
    fn = bw.gqa_causal_fwd if causal else bw.gqa_fwd
    o3, lse3 = fn(q3, k3, v.cuda())
    assert torch.equal(o3, o) and torch.equal(lse3, lse)
