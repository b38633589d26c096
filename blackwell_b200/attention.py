"""torch-tensor front end of the native attention library.

Mirrors the reference's Python entry points (base/baseline_gqa.py:57-59
``sdpa_gqa(q, k, v, scale)``, base/baseline_gqa_causal.py:61-65
``sdpa_gqa_causal``) and its CUDA launchers' argument meaning
(B, Hq, Hkv, S, G, scale; BHSD layout; hkv = hq // G).  Tensors are [B, H, S, D]
views; any view whose last dimension is contiguous works (a BSHD tensor
``x.transpose(1, 2)`` is passed through its strides, no copy).  Everything runs
in the native library on the current CUDA stream; there is no fallback path.
"""
from __future__ import annotations

import ctypes
import math

import torch

from . import _ffi


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _bhs(t: torch.Tensor):
    if t.dim() != 4 or t.stride(3) != 1:
        raise ValueError("expected a [B, H, S, D] tensor with a contiguous last dimension")
    return (t.stride(0), t.stride(1), t.stride(2))


def _check_inputs(q, k, v):
    for name, t in (("q", q), ("k", k), ("v", v)):
        if not t.is_cuda:
            raise ValueError(f"{name} must be a CUDA tensor")
        if t.dtype != torch.bfloat16:
            raise TypeError(f"{name} must be bfloat16, got {t.dtype}")
    B, Hq, Sq, D = q.shape
    Bk, Hkv, Skv, Dk = k.shape
    if v.shape != k.shape or Bk != B or Dk != D:
        raise ValueError(f"shape mismatch q={tuple(q.shape)} k={tuple(k.shape)} v={tuple(v.shape)}")
    if Hq % Hkv:
        raise ValueError("Hq must be a multiple of Hkv")
    return B, Hq, Hkv, Sq, Skv, D


def _strides(q, k, v, o):
    s = _ffi.BwStrides()
    for field, t in (("q", q), ("k", k), ("v", v), ("o", o)):
        getattr(s, field)[:] = _bhs(t)
    return ctypes.byref(s)


def _attn(q, k, v, scale, causal, out=None, lse=None, return_lse=True):
    B, Hq, Hkv, Sq, Skv, D = _check_inputs(q, k, v)
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    o = out if out is not None else torch.empty((B, Hq, Sq, D), dtype=torch.bfloat16, device=q.device)
    if return_lse and lse is None:
        lse = torch.empty((B, Hq, Sq), dtype=torch.float32, device=q.device)
    G = Hq // Hkv
    rc = _ffi.lib().bw_gqa_split_fwd(_ptr(q), _ptr(k), _ptr(v), _ptr(o), _ptr(lse), B, Hq, Hkv, Sq, Skv, G, D,
                                     float(scale), int(bool(causal)), _strides(q, k, v, o), _stream())
    _ffi.check(rc, "bw_gqa_split_fwd")
    return o, lse


def gqa_fwd(q, k, v, scale=None, out=None, lse=None):
    """Non-causal GQA forward -> (O bf16 [B,Hq,S,D], LSE fp32 [B,Hq,S])."""
    if q.shape[2] != k.shape[2]:
        raise ValueError("gqa_fwd needs Sq == Skv (use gqa_split_fwd)")
    return _attn(q, k, v, scale, False, out, lse)


def gqa_causal_fwd(q, k, v, scale=None, out=None, lse=None):
    """Causal GQA forward (key j visible to query i iff j <= i) -> (O, LSE)."""
    if q.shape[2] != k.shape[2]:
        raise ValueError("gqa_causal_fwd needs Sq == Skv")
    return _attn(q, k, v, scale, True, out, lse)


def gqa_split_fwd(q, k, v, scale=None, causal=False, out=None, lse=None):
    """GQA forward with Sq != Skv (the reference's split-length launcher) -> (O, LSE)."""
    return _attn(q, k, v, scale, causal, out, lse)


def gqa_causal_offset_fwd(q, k, v, q_offset, scale=None, out=None, lse=None):
    """Causal GQA of a chunk of queries against a longer key prefix: query row i
    is sequence position q_offset + i and sees keys j <= q_offset + i (chunked
    prefill; with Skv = q_offset + Sq the bottom-right-aligned mask) -> (O, LSE)."""
    B, Hq, Hkv, Sq, Skv, D = _check_inputs(q, k, v)
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    o = out if out is not None else torch.empty((B, Hq, Sq, D), dtype=torch.bfloat16, device=q.device)
    if lse is None:
        lse = torch.empty((B, Hq, Sq), dtype=torch.float32, device=q.device)
    rc = _ffi.lib().bw_gqa_causal_offset_fwd(_ptr(q), _ptr(k), _ptr(v), _ptr(o), _ptr(lse), B, Hq, Hkv, Sq, Skv,
                                             Hq // Hkv, D, float(scale), int(q_offset), _strides(q, k, v, o),
                                             _stream())
    _ffi.check(rc, "bw_gqa_causal_offset_fwd")
    return o, lse


def mha_fwd(q, k, v, scale=None, out=None, lse=None):
    """MHA forward (Hq == Hkv) -> (O, LSE)."""
    if q.shape[1] != k.shape[1]:
        raise ValueError("mha_fwd needs equal head counts")
    return _attn(q, k, v, scale, False, out, lse)


def sdpa_gqa(q, k, v, scale):
    """Drop-in for base/baseline_gqa.py:57-59: returns O only."""
    return _attn(q, k, v, scale, False, return_lse=False)[0]


def sdpa_gqa_causal(q, k, v, scale):
    """Drop-in for base/baseline_gqa_causal.py:61-65: returns O only."""
    return _attn(q, k, v, scale, True, return_lse=False)[0]


def decode_workspace_size(B, Hq, Hkv, D, total_tokens, chunk=0):
    return int(_ffi.lib().bw_gqa_decode_workspace_size(B, Hq, Hkv, D, int(total_tokens), int(chunk)))


def gqa_decode(q, k, v, kv_lens, kv_offsets, scale=None, chunk=0, workspace=None, out=None, lse=None):
    """Single-token split-KV GQA decode over ragged contiguous KV.

    q [B, Hq, D] bf16; k, v [total_tokens, Hkv, D] bf16; kv_lens int32 [B];
    kv_offsets int64 [B] (first token of each sequence).  Returns (O [B,Hq,D] bf16,
    LSE [B,Hq] fp32)."""
    for name, t in (("q", q), ("k", k), ("v", v)):
        if not t.is_cuda or t.dtype != torch.bfloat16 or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous bf16 CUDA tensor")
    if kv_lens.dtype != torch.int32 or kv_offsets.dtype != torch.int64:
        raise TypeError("kv_lens must be int32 and kv_offsets int64")
    B, Hq, D = q.shape
    total, Hkv, Dk = k.shape
    if Dk != D or v.shape != k.shape or kv_lens.numel() != B or kv_offsets.numel() != B:
        raise ValueError("shape mismatch")
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    need = decode_workspace_size(B, Hq, Hkv, D, total, chunk)
    if workspace is None:
        workspace = torch.empty(need, dtype=torch.uint8, device=q.device)
    o = out if out is not None else torch.empty((B, Hq, D), dtype=torch.bfloat16, device=q.device)
    if lse is None:
        lse = torch.empty((B, Hq), dtype=torch.float32, device=q.device)
    rc = _ffi.lib().bw_gqa_decode(_ptr(q), _ptr(k), _ptr(v), _ptr(kv_lens), _ptr(kv_offsets), _ptr(o), _ptr(lse),
                                  B, Hq, Hkv, D, int(total), float(scale), int(chunk), _ptr(workspace),
                                  workspace.numel() * workspace.element_size(), _stream())
    _ffi.check(rc, "bw_gqa_decode")
    return o, lse


def lse_combine(o_part, lse_part, out=None, lse=None):
    """Merge split partials: o_part fp32 [S, B, Hq, D], lse_part fp32 [S, B, Hq]."""
    S, B, Hq, D = o_part.shape
    if lse_part.shape != (S, B, Hq) or o_part.dtype != torch.float32 or lse_part.dtype != torch.float32:
        raise ValueError("bad partial shapes / dtypes")
    o_part, lse_part = o_part.contiguous(), lse_part.contiguous()
    o = out if out is not None else torch.empty((B, Hq, D), dtype=torch.bfloat16, device=o_part.device)
    if lse is None:
        lse = torch.empty((B, Hq), dtype=torch.float32, device=o_part.device)
    rc = _ffi.lib().bw_lse_combine(_ptr(o_part), _ptr(lse_part), S, B, Hq, D, _ptr(o), _ptr(lse), _stream())
    _ffi.check(rc, "bw_lse_combine")
    return o, lse


def packed_split_floats(B, Hq, D):
    """fp32 elements of one packed decode partial: O [B, Hq, D], then LSE [B, Hq],
    padded to a multiple of 4 (the layout bw_lse_combine_packed reads)."""
    return int(_ffi.lib().bw_decode_packed_split_floats(B, Hq, D))


def lse_combine_packed(parts, B, Hq, D, out=None, lse=None):
    """Merge packed partials: parts fp32 [S, packed_split_floats(B, Hq, D)]."""
    P = packed_split_floats(B, Hq, D)
    if parts.dim() != 2 or parts.shape[1] != P or parts.dtype != torch.float32 or not parts.is_contiguous():
        raise ValueError(f"parts must be a contiguous fp32 [splits, {P}] tensor")
    o = out if out is not None else torch.empty((B, Hq, D), dtype=torch.bfloat16, device=parts.device)
    if lse is None:
        lse = torch.empty((B, Hq), dtype=torch.float32, device=parts.device)
    rc = _ffi.lib().bw_lse_combine_packed(_ptr(parts), parts.shape[0], B, Hq, D, _ptr(o), _ptr(lse), _stream())
    _ffi.check(rc, "bw_lse_combine_packed")
    return o, lse


def stream_status() -> int:
    """Synchronise the current stream and return (and clear) its error code (each
    stream has its own error word on the device)."""
    return int(_ffi.lib().bw_stream_status(_stream()))


def set_option(key: int, value: int) -> None:
    _ffi.check(_ffi.lib().bw_set_option(key, int(value)), "bw_set_option")


def get_option(key: int) -> int:
    return int(_ffi.lib().bw_get_option(key))


def shard_plan(units: int, world: int, rank: int):
    b, e = ctypes.c_int64(), ctypes.c_int64()
    _ffi.check(_ffi.lib().bw_shard_plan(units, world, rank, ctypes.byref(b), ctypes.byref(e)), "bw_shard_plan")
    return b.value, e.value


def gqa_decode_partial(q, k, v, kv_lens, kv_offsets, scale=None, chunk=0, workspace=None, out=None, lse=None):
    """Split-KV decode over this GPU's keys only, leaving fp32 partials for a merge:
    returns (O fp32 [B,Hq,D] normalised by its own sum, LSE fp32 [B,Hq], -inf where
    a sequence has no local keys)."""
    for name, t in (("q", q), ("k", k), ("v", v)):
        if not t.is_cuda or t.dtype != torch.bfloat16 or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous bf16 CUDA tensor")
    if kv_lens.dtype != torch.int32 or kv_offsets.dtype != torch.int64:
        raise TypeError("kv_lens must be int32 and kv_offsets int64")
    B, Hq, D = q.shape
    total, Hkv, _ = k.shape
    o = out if out is not None else torch.empty((B, Hq, D), dtype=torch.float32, device=q.device)
    if lse is None:
        lse = torch.empty((B, Hq), dtype=torch.float32, device=q.device)
    if total == 0:  # no local keys at all: the neutral partial of the LSE merge
        o.zero_()
        lse.fill_(float("-inf"))
        return o, lse
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if workspace is None:
        workspace = torch.empty(decode_workspace_size(B, Hq, Hkv, D, total, chunk), dtype=torch.uint8,
                                device=q.device)
    rc = _ffi.lib().bw_gqa_decode_partial(_ptr(q), _ptr(k), _ptr(v), _ptr(kv_lens), _ptr(kv_offsets), _ptr(o),
                                          _ptr(lse), B, Hq, Hkv, D, int(total), float(scale), int(chunk),
                                          _ptr(workspace), workspace.numel() * workspace.element_size(), _stream())
    _ffi.check(rc, "bw_gqa_decode_partial")
    return o, lse


def gqa_decode_paged(q, k_cache, v_cache, block_table, kv_lens, scale=None, chunk=0, workspace=None, out=None,
                     lse=None):
    """Split-KV decode over a paged KV cache.

    q [B, Hq, D] bf16; k_cache / v_cache [num_pages, page_size, Hkv, D] bf16;
    block_table int32 [B, max_pages_per_seq]; kv_lens int32 [B].
    Returns (O [B, Hq, D] bf16, LSE [B, Hq] fp32)."""
    for name, t in (("q", q), ("k_cache", k_cache), ("v_cache", v_cache)):
        if not t.is_cuda or t.dtype != torch.bfloat16 or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous bf16 CUDA tensor")
    if block_table.dtype != torch.int32 or kv_lens.dtype != torch.int32 or not block_table.is_contiguous():
        raise TypeError("block_table and kv_lens must be contiguous int32")
    B, Hq, D = q.shape
    num_pages, page_size, Hkv, Dk = k_cache.shape
    if Dk != D or v_cache.shape != k_cache.shape or block_table.shape[0] != B or kv_lens.numel() != B:
        raise ValueError("shape mismatch")
    max_pages = block_table.shape[1]
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    bound = min(num_pages * page_size, B * max_pages * page_size)
    if workspace is None:
        workspace = torch.empty(decode_workspace_size(B, Hq, Hkv, D, bound, chunk), dtype=torch.uint8,
                                device=q.device)
    o = out if out is not None else torch.empty((B, Hq, D), dtype=torch.bfloat16, device=q.device)
    if lse is None:
        lse = torch.empty((B, Hq), dtype=torch.float32, device=q.device)
    rc = _ffi.lib().bw_gqa_decode_paged(_ptr(q), _ptr(k_cache), _ptr(v_cache), _ptr(block_table), _ptr(kv_lens),
                                        _ptr(o), _ptr(lse), B, Hq, Hkv, D, page_size, num_pages, max_pages,
                                        float(scale), int(chunk), _ptr(workspace),
                                        workspace.numel() * workspace.element_size(), _stream())
    _ffi.check(rc, "bw_gqa_decode_paged")
    return o, lse


def qk_norm_rope(x, cos_sin_cache, gamma=None, eps=1e-6, pos_offset=0, interleaved=False, out=None,
                 return_rstd=False):
    """QK-norm (RMSNorm over D, optional) + RoPE on a [B, H, S, D] bf16 tensor
    (the prologue of the reference's fused op).  Returns y (and rstd fp32 [B, H, S])."""
    if not x.is_cuda or x.dtype != torch.bfloat16 or x.stride(3) != 1:
        raise ValueError("x must be a bf16 CUDA [B, H, S, D] tensor with contiguous D")
    B, H, S, D = x.shape
    y = out if out is not None else torch.empty((B, H, S, D), dtype=torch.bfloat16, device=x.device)
    rstd = torch.empty((B, H, S), dtype=torch.float32, device=x.device) if return_rstd else None
    xs = (ctypes.c_int64 * 3)(*_bhs(x))
    ys = (ctypes.c_int64 * 3)(*_bhs(y))
    cache = cos_sin_cache.contiguous()
    g = gamma.contiguous() if gamma is not None else None
    rc = _ffi.lib().bw_qk_norm_rope(_ptr(x), _ptr(y), B, H, S, D, xs, ys, _ptr(cache), cache.shape[0], int(pos_offset),
                                    _ptr(g), float(eps), int(bool(interleaved)), _ptr(rstd), _stream())
    _ffi.check(rc, "bw_qk_norm_rope")
    return (y, rstd) if return_rstd else y


def gqa_fused_fwd(q, k, v, cos_sin_cache, q_gamma=None, k_gamma=None, eps=1e-6, pos_offset=0, interleaved=False,
                  scale=None, causal=False):
    """QK-norm + RoPE + GQA attention (the reference's fused op), BHSD contiguous.
    Returns (O, LSE, q_rstd, k_rstd)."""
    B, Hq, Hkv, S, _, D = _check_inputs(q, k, v)
    for t in (q, k, v):
        if not t.is_contiguous():
            raise ValueError("gqa_fused_fwd expects contiguous BHSD tensors")
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    ws = torch.empty(int(_ffi.lib().bw_gqa_fused_workspace_size(B, Hq, Hkv, S, D)), dtype=torch.uint8,
                     device=q.device)
    o = torch.empty_like(q)
    lse = torch.empty((B, Hq, S), dtype=torch.float32, device=q.device)
    qr = torch.empty((B, Hq, S), dtype=torch.float32, device=q.device)
    kr = torch.empty((B, Hkv, S), dtype=torch.float32, device=q.device)
    cache = cos_sin_cache.contiguous()
    rc = _ffi.lib().bw_gqa_fused_fwd(_ptr(q), _ptr(k), _ptr(v), _ptr(o), _ptr(lse), _ptr(cache),
                                     _ptr(q_gamma), _ptr(k_gamma), _ptr(qr), _ptr(kr), B, Hq, Hkv, S, Hq // Hkv, D,
                                     cache.shape[0], int(pos_offset), float(eps), int(bool(interleaved)),
                                     float(scale), int(bool(causal)), _ptr(ws), ws.numel(), _stream())
    _ffi.check(rc, "bw_gqa_fused_fwd")
    return o, lse, qr, kr


def _host_layout(t):
    """BW_LAYOUT_BHSD / BW_LAYOUT_BSHD for a contiguous host tensor seen as [B, H, S, D]."""
    B, H, S, D = t.shape
    st = t.stride()
    if st == (H * S * D, S * D, D, 1):
        return _ffi.BW_LAYOUT_BHSD
    if st == (S * H * D, D, H * D, 1):
        return _ffi.BW_LAYOUT_BSHD
    return None


def host_workspace_size(B, Hq, Hkv, S, D):
    """Device bytes `attention_from_host` needs for its copies of Q, K, V, O, LSE."""
    return int(_ffi.lib().bw_attn_fwd_host_workspace_size(B, Hq, Hkv, S, D))


def attention_from_host(q_host, k_host, v_host, o_host, lse_host=None, scale=None, causal=False, chunks=4,
                        workspace=None):
    """Attention forward on HOST tensors through `bw_attn_fwd_host`.

    q/k/v/o_host: [B, H, S, D] views of contiguous BHSD or BSHD host tensors
    (bf16; page-locked for the copies to overlap); lse_host: fp32 [B, Hq, S]
    or None.  The library cuts the work into `chunks` pieces and overlaps
    copy-in, the kernel and copy-out (causal: along the sequence, otherwise
    along the batch).  `workspace`: a uint8 CUDA tensor of at least
    `host_workspace_size(...)` bytes, reused across calls; allocated when None.
    Asynchronous like the other calls: synchronise the current stream before
    reading o_host / lse_host."""
    B, Hq, S, D = q_host.shape
    Hkv = k_host.shape[1]
    layout = _host_layout(q_host)
    if layout is None or any(_host_layout(t) != layout for t in (k_host, v_host, o_host)):
        raise ValueError("host tensors must be contiguous BHSD or BSHD, all in the same layout")
    for t in (q_host, k_host, v_host, o_host):
        if t.is_cuda or t.dtype != torch.bfloat16:
            raise ValueError("q/k/v/o_host must be bf16 host tensors")
    if lse_host is not None and (lse_host.is_cuda or lse_host.dtype != torch.float32 or not lse_host.is_contiguous()
                                 or tuple(lse_host.shape) != (B, Hq, S)):
        raise ValueError("lse_host must be a contiguous fp32 host tensor [B, Hq, S]")
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    need = host_workspace_size(B, Hq, Hkv, S, D)
    if workspace is None:
        workspace = torch.empty(need, dtype=torch.uint8, device=torch.device("cuda", torch.cuda.current_device()))
    rc = _ffi.lib().bw_attn_fwd_host(_ptr(q_host), _ptr(k_host), _ptr(v_host), _ptr(o_host), _ptr(lse_host),
                                     B, Hq, Hkv, S, D, float(scale), int(bool(causal)), layout, int(chunks),
                                     _ptr(workspace), workspace.numel(), _stream())
    _ffi.check(rc, "bw_attn_fwd_host")
    return o_host, lse_host


def mha_fwd_f32(q, k, v, scale=None, out=None, lse=None):
    """fp32 MHA forward at fp32 accuracy (the reference's mha_v3_tc: fp32 in / out
    and its 3xTF32 split), D = 64: Q K^T and P V each as three TF32 tensor-core
    products of hi / lo parts (split into a workspace):
    q, k, v [B, H, S, 64] float32 CUDA views with contiguous D.  Returns (O fp32, LSE)."""
    for name, t in (("q", q), ("k", k), ("v", v)):
        if not t.is_cuda or t.dtype != torch.float32 or t.dim() != 4 or t.stride(3) != 1:
            raise ValueError(f"{name} must be a float32 CUDA [B, H, S, D] tensor with contiguous D")
    B, H, S, D = q.shape
    if k.shape != q.shape or v.shape != q.shape:
        raise ValueError("q, k, v must have the same shape")
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    o = out if out is not None else torch.empty((B, H, S, D), dtype=torch.float32, device=q.device)
    if lse is None:
        lse = torch.empty((B, H, S), dtype=torch.float32, device=q.device)
    ws = torch.empty(int(_ffi.lib().bw_mha_f32_workspace_size(B, H, S, D)), dtype=torch.uint8, device=q.device)
    rc = _ffi.lib().bw_mha_fwd_f32(_ptr(q), _ptr(k), _ptr(v), _ptr(o), _ptr(lse), B, H, S, D, float(scale),
                                   _strides(q, k, v, o), _ptr(ws), ws.numel(), _stream())
    _ffi.check(rc, "bw_mha_fwd_f32")
    return o, lse
