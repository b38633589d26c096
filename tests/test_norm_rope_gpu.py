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


def test_fused_attention():
    import blackwell_b200 as bw
    B, Hq, Hkv, S, D = 1, 4, 2, 300, 128
    q, k, v = seeded_bf16((B, Hq, S, D), 51), seeded_bf16((B, Hkv, S, D), 52), seeded_bf16((B, Hkv, S, D), 53)
    cache = orc.rope_cache(S, D)
    g = torch.Generator().manual_seed(3)
    qg = (1 + 0.1 * torch.randn(D, generator=g)).float()
    kg = (1 + 0.1 * torch.randn(D, generator=g)).float()
    o, lse, qr, kr = bw.gqa_fused_fwd(q.cuda(), k.cuda(), v.cuda(), torch.from_numpy(cache).cuda(), qg.cuda(),
                                      kg.cuda(), causal=True)
    assert bw.stream_status() == 0
    q2, rq = orc.norm_rope_reference(q.float().numpy(), cache, qg.numpy(), 1e-6, 0, False)
    k2, rk = orc.norm_rope_reference(k.float().numpy(), cache, kg.numpy(), 1e-6, 0, False)
    ro, rl = orc.fp64_reference(q2, k2, v.float(), 1 / math.sqrt(D), causal=True)
    assert np.abs(o.float().cpu().numpy() - ro).max() <= O_TOL
    assert np.abs(lse.cpu().numpy() - rl).max() <= LSE_TOL
    np.testing.assert_allclose(qr.cpu().numpy(), rq, rtol=1e-5)
    np.testing.assert_allclose(kr.cpu().numpy(), rk, rtol=1e-5)
