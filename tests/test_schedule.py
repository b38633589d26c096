"""Host-side checks of the work schedules the prefill kernels and the host
pipeline use (restated from fmha_fwd3.cu and host_pipeline.cu, where they are
documented): the K/V ring order the producer loads in matches the positions
the two MMA issuers compute, causal work items weigh the same, and the host
pipeline's sequence chunks tile the sequence in 128-row steps."""
import pytest


def producer_order(n):
    """Producer load order for a segment of n key tiles: K0, K1, then V(j), K(j+2)."""
    seq = [("K", 0)] + ([("K", 1)] if n > 1 else [])
    for j in range(n):
        seq.append(("V", j))
        if j + 2 < n:
            seq.append(("K", j + 2))
    return seq


def pos_k(j):
    return j if j < 2 else 2 * j - 1


def pos_v(j, n):
    if n == 1:
        return 1
    return 2 + 2 * j if j <= n - 2 else 2 * n - 1


@pytest.mark.parametrize("n", range(1, 70))
def test_ring_positions_match_producer_order(n):
    seq = producer_order(n)
    assert len(seq) == 2 * n
    for i, (kind, j) in enumerate(seq):
        assert (pos_k(j) if kind == "K" else pos_v(j, n)) == i


@pytest.mark.parametrize("nqt,q_offset", [(32, 0), (31, 0), (1, 0), (16, 256), (9, 128)])
def test_causal_pairs_balance(nqt, q_offset):
    """Causal items pair query tiles (nqt-1-p, p): every item carries the same
    number of key tiles (one fewer for the middle tile of an odd count)."""
    per_tile = [min((q_offset + t * 128 + 127) // 128 + 1, 10 ** 9) for t in range(nqt)]
    weights = []
    for p in range((nqt + 1) // 2):
        a, b = nqt - 1 - p, p
        weights.append(per_tile[a] + (per_tile[b] if a != b else 0))
    full = [w for p, w in enumerate(weights) if nqt - 1 - p != p]
    assert len(set(full)) <= 1


@pytest.mark.parametrize("S,chunks", [(4096, 8), (320, 3), (1000, 8), (64, 4), (777, 32), (128, 1)])
def test_host_pipeline_sequence_chunks(S, chunks):
    """bw_attn_fwd_host cuts causal calls into <= chunks pieces whose bounds are
    multiples of 128 rows (the query offset of each piece) and end at S; the
    pieces shrink from first to last (weights nc .. 1), so the work left after
    the last copy-in is the smallest piece."""
    ntiles = (S + 127) // 128
    nc = min(chunks, 32, ntiles)
    wsum = nc * (nc + 1) // 2

    def bound(c):
        w = c * nc - c * (c - 1) // 2
        u = (w * ntiles + wsum // 2) // wsum
        return S if c == nc else min(u * 128, S)

    bounds = [bound(c) for c in range(nc + 1)]
    assert bounds[0] == 0 and bounds[-1] == S
    assert all(b % 128 == 0 for b in bounds if b < S)
    assert all(x <= y for x, y in zip(bounds, bounds[1:]))
    sizes = [y - x for x, y in zip(bounds, bounds[1:]) if y > x]
    assert sizes[-1] == min(sizes)
    if (S, chunks) == (4096, 8):
        assert [z // 128 for z in sizes] == [7, 6, 6, 4, 4, 2, 2, 1]
