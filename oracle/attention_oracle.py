"""CPU oracle for the GQA / MHA attention forward and the split-KV decode.

TEST INFRASTRUCTURE ONLY.  Nothing in the shipped library imports this module:
only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
(``cpu_baseline`` / ``--impl reference``) use it, and only as the checker or as
the timed CPU path of the reference, never as the thing measured on the GPU.

It restates, in numpy float64, the reference's own ground-truth functions:

* ``fp64_reference``        -- base/baseline_gqa.py:35-54 (non-causal GQA,
                               one (b, hq) head at a time, hkv = hq // G)
* ``fp64_reference`` with ``causal=True``
                            -- base/baseline_gqa_causal.py:35-58 (mask j > i
                               with ``triu(diagonal=1)``; top-left aligned)
* split lengths Sq != Skv   -- base/baseline_gqa_split.py:33-48
* ``fp64_attention``        -- base/baseline_mha.py:28-33 (MHA, G = 1)
* ``decode_reference``      -- no reference kernel exists for split-KV decode;
                               it is ``baseline_gqa_split.py:33-48`` applied per
                               sequence with Sq = 1, Skv = L_b.
* ``lse_combine_reference`` -- no reference implementation; the merge identity
                               O = sum_i e^{LSE_i - LSE*} O_i / sum_i e^{LSE_i - LSE*}.

The reference's CPU execution path (what ``bench.py --impl reference`` times)
is torch SDPA with ``enable_gqa=True``: ``sdpa_gqa`` (base/baseline_gqa.py:57-59),
``sdpa_gqa_causal`` (base/baseline_gqa_causal.py:61-65) and the split variant
(base/baseline_gqa_split.py:51-52).  ``sdpa_cpu`` below makes that same call on
CPU tensors.

Parity of this restatement is pinned by ``tests/test_oracle.py`` against golden
vectors produced by the reference's own functions (``tests/golden/make_golden.py``).
"""
from __future__ import annotations

import math

import numpy as np

LN2 = math.log(2.0)


def _as64(x) -> np.ndarray:
    if hasattr(x, "detach"):  # torch tensor
        x = x.detach().float().cpu().numpy()
    return np.asarray(x, dtype=np.float64)


def _row_attention(q64, k64, v64, scale, mask=None):
    """One head: scores = q k^T * scale, optional boolean mask (True = disallowed),
    LSE = logsumexp(scores), O = softmax(scores) v.  Mirrors the per-head body of
    base/baseline_gqa.py:45-53 / base/baseline_gqa_causal.py:50-57 in float64."""
    scores = (q64 @ k64.T) * scale
    if mask is not None:
        scores = np.where(mask, -np.inf, scores)
    mx = scores.max(axis=-1, keepdims=True)
    mx_safe = np.where(np.isfinite(mx), mx, 0.0)
    e = np.exp(scores - mx_safe)
    s = e.sum(axis=-1, keepdims=True)
    lse = (np.log(s) + mx_safe)[..., 0]
    out = (e / s) @ v64
    return out, lse


def fp64_reference(q, k, v, scale, causal=False):
    """Ground truth O (float32) and LSE (float32, natural log) for BHSD inputs.

    q: [B, Hq, Sq, D], k/v: [B, Hkv, Skv, D].  GQA routing hkv = hq // G with
    G = Hq // Hkv (base/baseline_gqa.py:42-46).  ``causal`` applies the mask
    j > i (base/baseline_gqa_causal.py:43-45, 53)."""
    q, k, v = _as64(q), _as64(k), _as64(v)
    B, Hq, Sq, D = q.shape
    Hkv, Skv = k.shape[1], k.shape[2]
    G = Hq // Hkv
    out = np.empty((B, Hq, Sq, D), dtype=np.float32)
    lse = np.empty((B, Hq, Sq), dtype=np.float32)
    mask = None
    if causal:
        mask = np.triu(np.ones((Sq, Skv), dtype=bool), k=1)
    for b in range(B):
        for hq in range(Hq):
            hkv = hq // G
            o, l = _row_attention(q[b, hq], k[b, hkv], v[b, hkv], scale, mask)
            out[b, hq] = o
            lse[b, hq] = l
    return out, lse


def fp64_rows(q, k, v, scale, causal, rows):
    """Exact float64 output for a subset of query rows.

    ``rows`` is an int array [R, 3] of (b, hq, i).  Every query row of attention
    is independent, so this is the same arithmetic as ``fp64_reference`` restricted
    to those rows (used at the full config sizes, where the all-rows oracle would
    take hours).  Returns O [R, D] float64 and LSE [R] float64."""
    q, k, v = _as64(q), _as64(k), _as64(v)
    Hq, Hkv = q.shape[1], k.shape[1]
    G = Hq // Hkv
    outs, lses = [], []
    for b, hq, i in np.asarray(rows):
        hkv = hq // G
        kk, vv = k[b, hkv], v[b, hkv]
        if causal:
            kk, vv = kk[: i + 1], vv[: i + 1]
        o, l = _row_attention(q[b, hq, i : i + 1], kk, vv, scale)
        outs.append(o[0])
        lses.append(l[0])
    return np.stack(outs), np.asarray(lses)


def fp64_attention(q, k, v, scale):
    """MHA ground truth (base/baseline_mha.py:28-33): softmax(q k^T * scale) v."""
    o, _ = fp64_reference(q, k, v, scale, causal=False)
    return o


def decode_reference(q, k, v, kv_lens, kv_offsets, scale):
    """Single-token GQA decode over ragged, contiguous per-sequence KV.

    q: [B, Hq, D]; k/v: [total_tokens, Hkv, D]; sequence b owns tokens
    [kv_offsets[b], kv_offsets[b] + kv_lens[b]).  Each sequence is the split-length
    reference (base/baseline_gqa_split.py:33-48) with Sq = 1, Skv = L_b.
    Returns O [B, Hq, D] float32, LSE [B, Hq] float32."""
    q, k, v = _as64(q), _as64(k), _as64(v)
    B, Hq, D = q.shape
    Hkv = k.shape[1]
    G = Hq // Hkv
    out = np.empty((B, Hq, D), dtype=np.float32)
    lse = np.empty((B, Hq), dtype=np.float32)
    for b in range(B):
        s0, L = int(kv_offsets[b]), int(kv_lens[b])
        for hq in range(Hq):
            hkv = hq // G
            o, l = _row_attention(q[b, hq][None], k[s0 : s0 + L, hkv], v[s0 : s0 + L, hkv], scale)
            out[b, hq] = o[0]
            lse[b, hq] = l[0]
    return out, lse


def lse_combine_reference(o_parts, lse_parts):
    """Merge split partials.  o_parts [S, ..., D] (each normalised by its own sum),
    lse_parts [S, ...] (natural log).  Returns (O, LSE) with
    LSE = LSE* + ln sum_i e^{LSE_i - LSE*},  O = sum_i e^{LSE_i - LSE} O_i.
    A split whose LSE is -inf (no keys) contributes nothing."""
    o = _as64(o_parts)
    l = _as64(lse_parts)
    lmax = l.max(axis=0)
    lmax_safe = np.where(np.isfinite(lmax), lmax, 0.0)
    w = np.exp(l - lmax_safe[None])
    tot = w.sum(axis=0)
    lse = np.log(tot) + lmax_safe
    out = (w[..., None] * o).sum(axis=0) / tot[..., None]
    return out.astype(np.float32), lse.astype(np.float32)


def sdpa_cpu(q, k, v, scale, causal=False):
    """The reference's CPU execution path: torch SDPA with enable_gqa on CPU tensors
    (base/baseline_gqa.py:57-59, base/baseline_gqa_causal.py:61-65).  Returns O only,
    like the reference's ``sdpa_gqa*`` functions."""
    import torch.nn.functional as F

    return F.scaled_dot_product_attention(q, k, v, scale=scale, enable_gqa=True, is_causal=causal)
