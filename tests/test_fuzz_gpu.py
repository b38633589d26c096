"""Randomised shapes for the attention forward and the decode (seeded, so every
run checks the same cases): sizes, head counts, causal flag, split lengths,
layouts and chunk sizes drawn at random, each checked against the oracle."""
import math

import numpy as np
import pytest
import torch

from oracle import attention_oracle as orc
from tests._util import LSE_TOL, O_TOL, seeded_bf16

pytestmark = pytest.mark.gpu

RNG = np.random.default_rng(2024)
PREFILL = []
for _ in range(16):
    Hkv = int(RNG.choice([1, 2, 3]))
    G = int(RNG.choice([1, 2, 3, 4, 5, 8]))
    Sq = int(RNG.integers(1, 420))
    Skv = Sq if RNG.random() < 0.6 else int(RNG.integers(1, 420))
    PREFILL.append((int(RNG.integers(1, 3)), Hkv * G, Hkv, Sq, Skv, int(RNG.choice([64, 128])),
                    bool(RNG.random() < 0.5), bool(RNG.random() < 0.5)))


@pytest.mark.parametrize("case", PREFILL, ids=lambda c: "x".join(map(str, c)))
def test_prefill_fuzz(case):
    import blackwell_b200 as bw
    B, Hq, Hkv, Sq, Skv, D, causal, bshd = case
    seed = abs(hash(case)) % 1000
    q = seeded_bf16((B, Sq, Hq, D) if bshd else (B, Hq, Sq, D), seed)
    k = seeded_bf16((B, Skv, Hkv, D) if bshd else (B, Hkv, Skv, D), seed + 1)
    v = seeded_bf16((B, Skv, Hkv, D) if bshd else (B, Hkv, Skv, D), seed + 2)
    if bshd:
        q, k, v = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
    o, lse = bw.gqa_split_fwd(q.cuda(), k.cuda(), v.cuda(), causal=causal)
    assert bw.stream_status() == 0
    ro, rl = orc.fp64_reference(q.float(), k.float(), v.float(), 1 / math.sqrt(D), causal=causal)
    assert np.abs(o.float().cpu().numpy() - ro).max() <= O_TOL
    assert np.abs(lse.cpu().numpy() - rl).max() <= LSE_TOL


DECODE = []
for _ in range(8):
    Hkv = int(RNG.choice([1, 2, 4, 8]))
    G = int(RNG.choice([1, 2, 4, 6, 8, 12, 16]))
    B = int(RNG.integers(1, 7))
    DECODE.append((B, Hkv * G, Hkv, int(RNG.choice([64, 128])), int(RNG.integers(1, 3000)),
                   int(RNG.choice([64, 192, 512, 1024]))))


@pytest.mark.parametrize("case", DECODE, ids=lambda c: "x".join(map(str, c)))
def test_decode_fuzz(case):
    import blackwell_b200 as bw
    B, Hq, Hkv, D, maxlen, chunk = case
    rng = np.random.default_rng(abs(hash(case)) % 1000)
    lens = rng.integers(1, maxlen + 1, B)
    offs = np.concatenate([[0], np.cumsum(lens)[:-1]]).astype(np.int64)
    total = int(lens.sum())
    q = seeded_bf16((B, Hq, D), 71)
    k = seeded_bf16((total, Hkv, D), 72)
    v = seeded_bf16((total, Hkv, D), 73)
    o, lse = bw.gqa_decode(q.cuda(), k.cuda(), v.cuda(), torch.from_numpy(lens.astype(np.int32)).cuda(),
                           torch.from_numpy(offs).cuda(), chunk=chunk)
    assert bw.stream_status() == 0
    ro, rl = orc.decode_reference(q.float(), k.float(), v.float(), lens, offs, 1 / math.sqrt(D))
    assert np.abs(o.float().cpu().numpy() - ro).max() <= O_TOL
    assert np.abs(lse.cpu().numpy() - rl).max() <= LSE_TOL
