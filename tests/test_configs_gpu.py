"""Parity at the full size of every BASELINE configuration that the benchmark
times (through the C ABI), against the fp64 oracle on the same bf16 bits.

* C4  split-KV decode B=64, Hq=64, Hkv=8, D=128, L_b ~ U[1024, 32768] (seed 42):
      all 4096 (b, hq) rows, contiguous KV and paged KV (page 16 and 64, pages in
      the benchmark's random physical order).  Reference semantics:
      base/baseline_gqa_split.py:33-48 per sequence with Sq = 1.
* C3  non-causal MHA B=8, H=16, S=2048, D=64 and D=128: 2048 random rows plus
      the tile-edge rows (base/baseline_mha.py:28-33).
* C5  causal GQA B=1, Hq=64, Hkv=8, S=131072, D=128, cut into per-rank shards of
      whole KV groups exactly as the benchmark cuts it for 2, 4 and 8 ranks
      (inputs drawn per rank from seed 42 + rank); 8 ranks = one KV group per
      shard at S=131072 (base/baseline_gqa_causal.py:35-58).

Bar: max-abs error <= 2e-2 on bf16 O and <= 1e-3 on LSE."""
import math

import numpy as np
import pytest
import torch

from oracle import attention_oracle as orc
from tests._util import LSE_TOL, O_TOL

pytestmark = pytest.mark.gpu

C4 = dict(B=64, Hq=64, Hkv=8, D=128)


def _c4_lens():
    return torch.randint(1024, 32769, (C4["B"],), generator=torch.Generator().manual_seed(42))


def _check_decode_rows(q, k_of, v_of, lens, o, lse):
    """All (b, hq) rows of a decode against the oracle; k_of(b) / v_of(b) give
    sequence b's keys [L_b, Hkv, D] (on the GPU, widened on the host one
    sequence at a time)."""
    B, Hq, D = q.shape
    scale = 1 / math.sqrt(D)
    eo = el = 0.0
    oc, lc = o.float().cpu().numpy(), lse.cpu().numpy()
    for b in range(B):
        L = int(lens[b])
        ro, rl = orc.decode_reference(q[b:b + 1], k_of(b), v_of(b), [L], [0], scale)
        eo = max(eo, float(np.abs(oc[b] - ro[0]).max()))
        el = max(el, float(np.abs(lc[b] - rl[0]).max()))
    assert eo <= O_TOL, eo
    assert el <= LSE_TOL, el


def test_c4_decode_all_rows():
    import blackwell_b200 as bw
    B, Hq, Hkv, D = (C4[k] for k in ("B", "Hq", "Hkv", "D"))
    lens = _c4_lens()
    total = int(lens.sum())
    assert total == 955232
    offs = torch.cumsum(lens, 0) - lens
    g = torch.Generator(device="cuda").manual_seed(42)
    q = torch.randn(B, Hq, D, generator=g, device="cuda").bfloat16()
    k = torch.randn(total, Hkv, D, generator=g, device="cuda").bfloat16()
    v = torch.randn(total, Hkv, D, generator=g, device="cuda").bfloat16()
    o, lse = bw.gqa_decode(q, k, v, lens.int().cuda(), offs.long().cuda())
    assert bw.stream_status() == 0
    offs_l = offs.tolist()
    _check_decode_rows(q, lambda b: k[offs_l[b]:offs_l[b] + int(lens[b])], lambda b: v[offs_l[b]:offs_l[b] + int(lens[b])],
                       lens, o, lse)


@pytest.mark.parametrize("page_size", [16, 64])
def test_c4_decode_paged_all_rows(page_size):
    import blackwell_b200 as bw
    B, Hq, Hkv, D = (C4[k] for k in ("B", "Hq", "Hkv", "D"))
    lens = _c4_lens()
    pages = (lens + page_size - 1) // page_size
    num_pages, max_pages = int(pages.sum()), int(pages.max())
    perm = torch.randperm(num_pages, generator=torch.Generator().manual_seed(42)).int()
    bt = torch.full((B, max_pages), -1, dtype=torch.int32)
    start = 0
    for b in range(B):
        bt[b, :pages[b]] = perm[start:start + pages[b]]
        start += int(pages[b])
    g = torch.Generator(device="cuda").manual_seed(42)
    q = torch.randn(B, Hq, D, generator=g, device="cuda").bfloat16()
    kc = torch.randn(num_pages, page_size, Hkv, D, generator=g, device="cuda").bfloat16()
    vc = torch.randn(num_pages, page_size, Hkv, D, generator=g, device="cuda").bfloat16()
    bt_d = bt.cuda()
    o, lse = bw.attention.gqa_decode_paged(q, kc, vc, bt_d, lens.int().cuda())
    assert bw.stream_status() == 0

    def gather(cache, b):
        L = int(lens[b])
        tok = torch.arange(L, device="cuda")
        return cache[bt_d[b, tok // page_size].long(), tok % page_size]

    _check_decode_rows(q, lambda b: gather(kc, b), lambda b: gather(vc, b), lens, o, lse)


@pytest.mark.parametrize("D", [64, 128])
def test_c3_mha_full_size_rows(D):
    import blackwell_b200 as bw
    B, H, S = 8, 16, 2048
    g = torch.Generator(device="cuda").manual_seed(42)
    q = torch.randn(B, H, S, D, generator=g, device="cuda").bfloat16()
    k = torch.randn(B, H, S, D, generator=g, device="cuda").bfloat16()
    v = torch.randn(B, H, S, D, generator=g, device="cuda").bfloat16()
    o, lse = bw.mha_fwd(q, k, v)
    assert bw.stream_status() == 0
    rng = np.random.default_rng(D)
    rows = np.stack([rng.integers(0, B, 2048), rng.integers(0, H, 2048), rng.integers(0, S, 2048)], 1)
    edges = np.array([0, 1, 127, 128, 129, 255, 256, 1023, 1024, 2046, 2047])
    extra = np.stack([rng.integers(0, B, len(edges)), rng.integers(0, H, len(edges)), edges], 1)
    rows = np.concatenate([rows, extra])
    ro, rl = orc.fp64_rows(q, k, v, 1 / math.sqrt(D), False, rows)
    oc, lc = o.float().cpu().numpy(), lse.cpu().numpy()
    got_o = oc[rows[:, 0], rows[:, 1], rows[:, 2]]
    got_l = lc[rows[:, 0], rows[:, 1], rows[:, 2]]
    assert np.abs(got_o - ro).max() <= O_TOL
    assert np.abs(got_l - rl).max() <= LSE_TOL


@pytest.mark.parametrize("world", [2, 4, 8])
def test_c5_rank_shards(world):
    """Each rank's shard of C5 as the benchmark cuts it (whole KV groups, inputs
    from seed 42 + rank), run one after another on one GPU; 48 rows per shard
    including the first and last tiles."""
    import blackwell_b200 as bw
    from blackwell_b200.distributed import unit_range
    Hq, Hkv, S, D = 64, 8, 131072, 128
    G = Hq // Hkv
    for rank in range(world):
        g0, g1 = unit_range(Hkv, world, rank)
        ng = g1 - g0
        gen = torch.Generator(device="cuda").manual_seed(42 + rank)
        q = torch.randn(1, ng * G, S, D, generator=gen, device="cuda").bfloat16()
        k = torch.randn(1, ng, S, D, generator=gen, device="cuda").bfloat16()
        v = torch.randn(1, ng, S, D, generator=gen, device="cuda").bfloat16()
        o, lse = bw.gqa_causal_fwd(q, k, v)
        assert bw.stream_status() == 0
        rng = np.random.default_rng(100 * world + rank)
        n = 48
        rows = np.stack([np.zeros(n, int), rng.integers(0, ng * G, n), rng.integers(0, S, n)], 1)
        rows[:6, 2] = [0, 127, 128, S - 129, S - 128, S - 1]
        ro, rl = orc.fp64_rows(q, k, v, 1 / math.sqrt(D), True, rows)
        got_o = o[0, rows[:, 1], rows[:, 2]].float().cpu().numpy()
        got_l = lse[0, rows[:, 1], rows[:, 2]].cpu().numpy()
        assert np.abs(got_o - ro).max() <= O_TOL, (world, rank)
        assert np.abs(got_l - rl).max() <= LSE_TOL, (world, rank)
        del q, k, v, o, lse
        torch.cuda.empty_cache()
