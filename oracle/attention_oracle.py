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


def fp64_rows(q, k, v, scale, causal, rows, q_offset=0):
    """Exact float64 output for a subset of query rows.

    ``rows`` is an int array [R, 3] of (b, hq, i).  Every query row of attention
    is independent, so this is the same arithmetic as ``fp64_reference`` restricted
    to those rows (used at the full config sizes, where the all-rows oracle would
    take hours).  ``q_offset`` (causal only) places query row i at sequence
    position q_offset + i, so it sees keys j <= q_offset + i (the chunked-prefill
    extension; 0 is the reference's top-left alignment).  Only the query rows
    asked for and the key / value heads they read are widened to float64 (one
    (b, kv head) at a time), so inputs of several GB stay in their own dtype.
    Returns O [R, D] float64 and LSE [R] float64."""
    rows = np.asarray(rows)
    Hq, Hkv = q.shape[1], k.shape[1]
    G = Hq // Hkv
    outs = np.empty((len(rows), q.shape[-1]))
    lses = np.empty(len(rows))
    kv_of = rows[:, 0] * Hkv + rows[:, 1] // G
    for key in np.unique(kv_of):
        b, hkv = divmod(int(key), Hkv)
        sel = np.nonzero(kv_of == key)[0]
        kk, vv = _as64(k[b, hkv]), _as64(v[b, hkv])
        for r in sel:
            hq, i = int(rows[r, 1]), int(rows[r, 2])
            lim = q_offset + i + 1 if causal else kk.shape[0]
            o, l = _row_attention(_as64(q[b, hq, i : i + 1]), kk[:lim], vv[:lim], scale)
            outs[r] = o[0]
            lses[r] = l[0]
    return outs, lses


def fp64_attention(q, k, v, scale):
    """MHA ground truth (base/baseline_mha.py:28-33): softmax(q k^T * scale) v."""
    o, _ = fp64_reference(q, k, v, scale, causal=False)
    return o


def decode_reference(q, k, v, kv_lens, kv_offsets, scale):
    """Single-token GQA decode over ragged, contiguous per-sequence KV.

    q: [B, Hq, D]; k/v: [total_tokens, Hkv, D]; sequence b owns tokens
    [kv_offsets[b], kv_offsets[b] + kv_lens[b]).  Each sequence is the split-length
    reference (base/baseline_gqa_split.py:33-48) with Sq = 1, Skv = L_b; the G
    query heads that share a KV head are evaluated together (independent rows of
    the same matrix product).  Only one sequence's keys are widened to float64 at
    a time, so k / v may be large tensors in their own dtype.
    Returns O [B, Hq, D] float32, LSE [B, Hq] float32."""
    B, Hq, D = q.shape
    Hkv = k.shape[1]
    G = Hq // Hkv
    out = np.empty((B, Hq, D), dtype=np.float32)
    lse = np.empty((B, Hq), dtype=np.float32)
    for b in range(B):
        s0, L = int(kv_offsets[b]), int(kv_lens[b])
        qb = _as64(q[b])
        kb, vb = _as64(k[s0 : s0 + L]), _as64(v[s0 : s0 + L])
        for hkv in range(Hkv):
            o, l = _row_attention(qb[hkv * G : (hkv + 1) * G], kb[:, hkv], vb[:, hkv], scale)
            out[b, hkv * G : (hkv + 1) * G] = o
            lse[b, hkv * G : (hkv + 1) * G] = l
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


def _bf16_round(x):
    """Round float32 values to bfloat16 (nearest even) and widen back to float32."""
    import torch

    return torch.from_numpy(np.asarray(x, dtype=np.float32)).bfloat16().float().numpy()


def norm_rope_reference(x, cache, gamma, eps, pos_offset, interleaved):
    """QK-norm + RoPE of the reference's fused op, restated from
    src/SM103/attention/GQA_fused_sm103.cu:59-104 (norm_rope_tile) with the same
    rounding points: fp32 math, bf16 after the norm, bf16 after the rotation.
    x: [B, H, S, D] (bf16 values as float32); cache: fp32 [L, D] (cos | sin).
    Returns (y [B, H, S, D] float32 holding bf16 values, rstd [B, H, S] float32)."""
    x = np.asarray(x, dtype=np.float32)
    B, H, S, D = x.shape
    half = D // 2
    rstd = np.zeros((B, H, S), np.float32)
    if gamma is not None:
        ss = (x.astype(np.float32) ** 2).sum(-1, dtype=np.float32)
        rstd = (1.0 / np.sqrt(ss / np.float32(D) + np.float32(eps))).astype(np.float32)
        x = _bf16_round(x * rstd[..., None] * np.asarray(gamma, np.float32))
    y = x.copy()
    L = cache.shape[0]
    for s in range(S):
        pos = s + pos_offset
        if not (0 <= pos < L):
            continue
        c = cache[pos, :half].astype(np.float32)
        sn = cache[pos, half:].astype(np.float32)
        if interleaved:
            a, b = x[:, :, s, 0::2], x[:, :, s, 1::2]
            y[:, :, s, 0::2] = a * c - b * sn
            y[:, :, s, 1::2] = a * sn + b * c
        else:
            a, b = x[:, :, s, :half], x[:, :, s, half:]
            y[:, :, s, :half] = a * c - b * sn
            y[:, :, s, half:] = a * sn + b * c
    return _bf16_round(y), rstd


def rope_cache(max_pos, D, theta=10000.0):
    """fp32 cos|sin cache [max_pos, D] in the reference's layout (cos in [0, D/2),
    sin in [D/2, D)) with the standard inverse-frequency schedule theta^(-2i/D)."""
    half = D // 2
    inv = theta ** (-np.arange(half, dtype=np.float64) * 2.0 / D)
    ang = np.arange(max_pos, dtype=np.float64)[:, None] * inv[None]
    return np.concatenate([np.cos(ang), np.sin(ang)], axis=1).astype(np.float32)
