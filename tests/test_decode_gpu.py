"""Split-KV decode and LSE-combine parity (through the C ABI)."""
import math

import numpy as np
import pytest
import torch

from oracle import attention_oracle as orc
from tests._util import LSE_TOL, O_TOL, bf16_from_bits, seeded_bf16

pytestmark = pytest.mark.gpu


def _decode(q, k, v, lens, chunk=0):
    import blackwell_b200 as bw
    lens = np.asarray(lens)
    offs = np.concatenate([[0], np.cumsum(lens)[:-1]]).astype(np.int64)
    o, lse = bw.gqa_decode(q.cuda(), k.cuda(), v.cuda(), torch.from_numpy(lens.astype(np.int32)).cuda(),
                           torch.from_numpy(offs).cuda(), chunk=chunk)
    assert bw.stream_status() == 0
    return o.float().cpu().numpy(), lse.cpu().numpy(), offs


@pytest.mark.parametrize("chunk", [0, 64, 256])
def test_decode_golden(golden, chunk):
    g = golden("decode_d128")
    q, k, v = (bf16_from_bits(g[n]) for n in ("q_bf16", "k_bf16", "v_bf16"))
    o, lse, _ = _decode(q, k, v, g["kv_lens"], chunk)
    assert np.abs(o - g["o_fp64"]).max() <= O_TOL
    assert np.abs(lse - g["lse_fp64"]).max() <= LSE_TOL


@pytest.mark.parametrize("B,Hq,Hkv,D,maxlen,chunk", [
    (5, 64, 8, 128, 3000, 1024), (3, 8, 8, 64, 700, 128), (4, 16, 1, 128, 2100, 512), (2, 12, 4, 64, 200, 64)])
def test_decode_ragged(B, Hq, Hkv, D, maxlen, chunk):
    rng = np.random.default_rng(B * 1000 + D)
    lens = rng.integers(1, maxlen + 1, B)
    lens[0] = 1
    total = int(lens.sum())
    q = seeded_bf16((B, Hq, D), 11)
    k = seeded_bf16((total, Hkv, D), 12)
    v = seeded_bf16((total, Hkv, D), 13)
    o, lse, offs = _decode(q, k, v, lens, chunk)
    ro, rl = orc.decode_reference(q.float(), k.float(), v.float(), lens, offs, 1 / math.sqrt(D))
    assert np.abs(o - ro).max() <= O_TOL
    assert np.abs(lse - rl).max() <= LSE_TOL


def test_decode_empty_sequence_gives_zero():
    q = seeded_bf16((2, 8, 128), 1)
    k = seeded_bf16((100, 1, 128), 2)
    v = seeded_bf16((100, 1, 128), 3)
    o, lse, _ = _decode(q, k, v, [0, 100])
    assert np.all(o[0] == 0) and np.all(np.isneginf(lse[0]))
    ro, rl = orc.decode_reference(q[1:].float(), k.float(), v.float(), [100], [0], 1 / math.sqrt(128))
    assert np.abs(o[1] - ro[0]).max() <= O_TOL


@pytest.mark.parametrize("splits", [1, 3, 64])
def test_lse_combine_kernel(splits):
    import blackwell_b200 as bw
    rng = np.random.default_rng(splits)
    B, Hq, D = 3, 5, 128
    op = rng.standard_normal((splits, B, Hq, D)).astype(np.float32)
    lp = (rng.standard_normal((splits, B, Hq)) * 3).astype(np.float32)
    if splits > 1:
        lp[0, 0, 0] = -np.inf
    o, lse = bw.lse_combine(torch.from_numpy(op).cuda(), torch.from_numpy(lp).cuda())
    ro, rl = orc.lse_combine_reference(op, lp)
    assert np.abs(o.float().cpu().numpy() - ro).max() <= O_TOL
    assert np.abs(lse.cpu().numpy() - rl).max() <= 1e-5


@pytest.mark.parametrize("pieces", [1, 2, 3])
def test_decode_partial_pieces_merge(pieces):
    """Keys of every sequence split into `pieces` (as across GPUs): fp32 partials from
    bw_gqa_decode_partial, merged by bw_lse_combine, equal the full decode."""
    import blackwell_b200 as bw
    from blackwell_b200.distributed import split_sequences
    B, Hq, Hkv, D = 5, 32, 4, 128
    lens = np.array([1, 2, 700, 1500, 64])
    offs = np.concatenate([[0], np.cumsum(lens)[:-1]])
    q = seeded_bf16((B, Hq, D), 21)
    k = seeded_bf16((int(lens.sum()), Hkv, D), 22)
    v = seeded_bf16((int(lens.sum()), Hkv, D), 23)
    os_, ls_ = [], []
    for r in range(pieces):
        loc, st = split_sequences(lens, pieces, r)
        rows = np.concatenate([np.arange(offs[b] + st[b], offs[b] + st[b] + loc[b]) for b in range(B)]).astype(np.int64)
        lo = np.concatenate([[0], np.cumsum(loc)[:-1]]).astype(np.int64)
        o, l = bw.attention.gqa_decode_partial(q.cuda(), k[rows].cuda().contiguous(), v[rows].cuda().contiguous(),
                                               torch.from_numpy(loc).cuda(), torch.from_numpy(lo).cuda(), chunk=128)
        os_.append(o)
        ls_.append(l)
    o, lse = bw.lse_combine(torch.stack(os_), torch.stack(ls_))
    assert bw.stream_status() == 0
    ro, rl = orc.decode_reference(q.float(), k.float(), v.float(), lens, offs, 1 / math.sqrt(D))
    assert np.abs(o.float().cpu().numpy() - ro).max() <= O_TOL
    assert np.abs(lse.cpu().numpy() - rl).max() <= LSE_TOL


@pytest.mark.parametrize("page_size,D", [(8, 128), (16, 128), (32, 128), (64, 128), (128, 128), (256, 128),
                                         (16, 64), (64, 64)])
def test_decode_paged(page_size, D):
    """Paged KV cache: pages in a random physical order, unused block-table
    entries set to -1, partial last pages; against the oracle on the gathered
    contiguous keys."""
    import blackwell_b200 as bw
    rng = np.random.default_rng(page_size)
    B, Hq, Hkv = 4, 32, 4
    lens = np.array([1, page_size + 3, 1100, 2 * page_size])
    pages_per = (lens + page_size - 1) // page_size
    max_pages = int(pages_per.max()) + 2
    num_pages = int(pages_per.sum()) + 5
    perm = rng.permutation(num_pages)
    bt = -np.ones((B, max_pages), np.int32)
    used = 0
    for b in range(B):
        bt[b, :pages_per[b]] = perm[used:used + pages_per[b]]
        used += pages_per[b]
    q = seeded_bf16((B, Hq, D), 31)
    kc = seeded_bf16((num_pages, page_size, Hkv, D), 32)
    vc = seeded_bf16((num_pages, page_size, Hkv, D), 33)
    o, lse = bw.attention.gqa_decode_paged(q.cuda(), kc.cuda(), vc.cuda(), torch.from_numpy(bt).cuda(),
                                           torch.from_numpy(lens.astype(np.int32)).cuda(), chunk=128)
    assert bw.stream_status() == 0
    # gather each sequence's tokens into one contiguous [total, Hkv, D] for the oracle
    ks, vs = [], []
    for b in range(B):
        toks = np.arange(lens[b])
        pg, sl = bt[b, toks // page_size], toks % page_size
        ks.append(kc[pg, sl])
        vs.append(vc[pg, sl])
    k = torch.cat(ks).float()
    v = torch.cat(vs).float()
    offs = np.concatenate([[0], np.cumsum(lens)[:-1]])
    ro, rl = orc.decode_reference(q.float(), k, v, lens, offs, 1 / math.sqrt(D))
    assert np.abs(o.float().cpu().numpy() - ro).max() <= O_TOL
    assert np.abs(lse.cpu().numpy() - rl).max() <= LSE_TOL


@pytest.mark.parametrize("entry", ["workspace", "static"])
def test_decode_overlapping_offsets_overflow_is_reported(entry):
    """Sequences that share rows through overlapping offsets can need more
    partials than a workspace sized from total_tokens holds.  The call must not
    read or write past the workspace: it writes empty rows (O = 0, LSE = -inf)
    and reports BW_ERR_WORKSPACE; the next call on the stream is clean."""
    import ctypes
    import blackwell_b200 as bw
    from blackwell_b200 import _ffi
    lib = _ffi.lib()
    B, Hq, Hkv, D, total, chunk = 4, 16, 2, 128, 4096, 64
    q = seeded_bf16((B, Hq, D), 41).cuda()
    k = seeded_bf16((total, Hkv, D), 42).cuda()
    v = seeded_bf16((total, Hkv, D), 43).cuda()
    lens = torch.full((B,), total, dtype=torch.int32, device="cuda")      # every sequence = all rows
    offs = torch.zeros(B, dtype=torch.int64, device="cuda")
    o = torch.full((B, Hq, D), 7.0, dtype=torch.bfloat16, device="cuda")
    lse = torch.zeros(B, Hq, dtype=torch.float32, device="cuda")
    P = lambda t: ctypes.c_void_p(t.data_ptr())
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    if entry == "workspace":
        n = lib.bw_gqa_decode_workspace_size(B, Hq, Hkv, D, total, chunk)
        guard = 1 << 20
        ws = torch.full((n + guard,), 0xAB, dtype=torch.uint8, device="cuda")
        rc = lib.bw_gqa_decode(P(q), P(k), P(v), P(lens), P(offs), P(o), P(lse), B, Hq, Hkv, D, total,
                               1 / math.sqrt(D), chunk, P(ws), n, stream)
    else:
        rc = lib.bw_gqa_decode_static(P(q), P(k), P(v), P(lens), P(offs), P(o), P(lse), B, Hq, Hkv, D, total,
                                      1 / math.sqrt(D), chunk, stream)
    assert rc == 0
    assert lib.bw_stream_status(stream) == _ffi.BW_ERR_WORKSPACE
    assert torch.all(o == 0) and torch.all(torch.isneginf(lse))
    if entry == "workspace":
        assert torch.all(ws[n:] == 0xAB)          # nothing written past the workspace
    # the same sequences without overlap fit and decode correctly afterwards
    o2, l2, _ = _decode(q.cpu(), k.cpu(), v.cpu(), [1024, 1024, 1024, 1024])
    ro, rl = orc.decode_reference(q.float().cpu(), k.float().cpu(), v.float().cpu(), [1024] * 4,
                                  [0, 1024, 2048, 3072], 1 / math.sqrt(D))
    assert np.abs(o2 - ro).max() <= O_TOL
    assert np.abs(l2 - rl).max() <= LSE_TOL
