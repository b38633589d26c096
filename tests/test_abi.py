"""C-ABI checks that need no GPU: the library loads, exports every symbol the
header declares, and rejects bad arguments before touching the device."""
import ctypes
import re
from pathlib import Path

import pytest

from blackwell_b200 import _ffi

HEADER = Path(__file__).resolve().parent.parent / "include" / "bw_attn.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"BW_API\s+[\w\s\*]*?\b(bw_\w+)\s*\(", text)))


def test_header_declares_the_boundary():
    syms = declared_symbols()
    for s in ["bw_gqa_fwd", "bw_gqa_causal_fwd", "bw_gqa_split_fwd", "bw_mha_fwd", "bw_gqa_decode",
              "bw_lse_combine", "bw_stream_status"]:
        assert s in syms


def test_library_exports_every_declared_symbol():
    lib = _ffi.lib()
    for s in declared_symbols():
        assert hasattr(lib, s), s
    assert set(declared_symbols()) <= set(_ffi.SIGNATURES)


def test_version_and_strerror():
    assert b"sm_100a" in _ffi.lib().bw_version()
    for code in range(8):
        assert _ffi.strerror(code)
    assert _ffi.strerror(99) == "unknown error"


def test_argument_validation_without_gpu():
    lib = _ffi.lib()
    p = ctypes.c_void_p(0x100000)
    none = ctypes.c_void_p(0)
    # NULL tensor
    assert lib.bw_gqa_fwd(none, p, p, p, None, 1, 8, 2, 128, 4, 64, 0.125, None, None) == _ffi.BW_ERR_NULL
    # unsupported head dim, inconsistent G, bad scale
    assert lib.bw_gqa_fwd(p, p, p, p, None, 1, 8, 2, 128, 4, 96, 0.1, None, None) == _ffi.BW_ERR_SHAPE
    assert lib.bw_gqa_fwd(p, p, p, p, None, 1, 8, 2, 128, 3, 64, 0.1, None, None) == _ffi.BW_ERR_SHAPE
    assert lib.bw_gqa_causal_fwd(p, p, p, p, None, 1, 8, 2, 128, 4, 64, -1.0, None, None) == _ffi.BW_ERR_SHAPE
    assert lib.bw_gqa_split_fwd(p, p, p, p, None, 1, 8, 2, 0, 5, 4, 64, 0.1, 0, None, None) == _ffi.BW_ERR_SHAPE
    # misaligned pointer / stride
    odd = ctypes.c_void_p(0x100002)
    assert lib.bw_mha_fwd(odd, p, p, p, None, 1, 4, 128, 64, 0.1, None, None) == _ffi.BW_ERR_ALIGN
    st = _ffi.BwStrides()
    for f in ("q", "k", "v", "o"):
        getattr(st, f)[:] = (4 * 128 * 64, 128 * 64, 60)
    assert lib.bw_mha_fwd(p, p, p, p, None, 1, 4, 128, 64, 0.1, ctypes.byref(st), None) == _ffi.BW_ERR_ALIGN
    # decode: G > 16, chunk not a multiple of 64, workspace too small
    i64 = ctypes.c_void_p(0x100000)
    assert lib.bw_gqa_decode(p, p, p, i64, i64, p, None, 2, 64, 2, 128, 100, 0.1, 0, p, 1 << 30, None) == \
        _ffi.BW_ERR_SHAPE
    assert lib.bw_gqa_decode(p, p, p, i64, i64, p, None, 2, 16, 2, 128, 100, 0.1, 100, p, 1 << 30, None) == \
        _ffi.BW_ERR_SHAPE
    assert lib.bw_gqa_decode(p, p, p, i64, i64, p, None, 2, 16, 2, 128, 100, 0.1, 0, p, 16, None) == \
        _ffi.BW_ERR_WORKSPACE
    assert lib.bw_lse_combine(None, None, 1, 1, 1, 64, None, None, None) == _ffi.BW_ERR_NULL


def test_decode_workspace_size_formula():
    lib = _ffi.lib()
    B, Hq, Hkv, D, T, ch = 64, 64, 8, 128, 1_000_000, 1024
    parts = Hkv * ((T + ch - 1) // ch + B)
    G = Hq // Hkv
    a256 = lambda x: (x + 255) // 256 * 256
    assert lib.bw_gqa_decode_workspace_size(B, Hq, Hkv, D, T, ch) == a256((B + 1) * 4) + a256(parts * G * 4) + \
        parts * G * D * 4
    assert lib.bw_gqa_decode_workspace_size(B, Hq, Hkv, D, T, 0) == lib.bw_gqa_decode_workspace_size(B, Hq, Hkv, D, T,
                                                                                                       1024)


def test_options_roundtrip():
    lib = _ffi.lib()
    old = lib.bw_get_option(_ffi.BW_OPT_TIMEOUT_NS)
    assert lib.bw_set_option(_ffi.BW_OPT_TIMEOUT_NS, 12345) == 0
    assert lib.bw_get_option(_ffi.BW_OPT_TIMEOUT_NS) == 12345
    assert lib.bw_set_option(_ffi.BW_OPT_TIMEOUT_NS, 0) == _ffi.BW_ERR_SHAPE
    lib.bw_set_option(_ffi.BW_OPT_TIMEOUT_NS, old)
    assert lib.bw_set_option(999, 1) == _ffi.BW_ERR_SHAPE


@pytest.mark.parametrize("units,world", [(32, 1), (32, 8), (7, 3), (0, 4), (5, 8)])
def test_shard_plan_partitions(units, world):
    from blackwell_b200 import shard_plan
    spans = [shard_plan(units, world, r) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == units
    for (a, b), (c, d) in zip(spans, spans[1:]):
        assert b == c and a <= b
    sizes = [e - b for b, e in spans]
    assert max(sizes) - min(sizes) <= 1


def test_package_exports():
    import blackwell_b200 as bw
    for name in ["gqa_fwd", "gqa_causal_fwd", "gqa_split_fwd", "mha_fwd", "gqa_decode", "gqa_decode_paged",
                 "gqa_decode_partial", "lse_combine", "qk_norm_rope", "gqa_fused_fwd", "sdpa_gqa", "sdpa_gqa_causal",
                 "stream_status", "set_option", "get_option", "shard_plan", "decode_workspace_size",
                 "attention_from_host", "gqa_causal_offset_fwd", "host_workspace_size"]:
        assert callable(getattr(bw, name)), name


def test_new_entry_points_validate_without_gpu():
    """The host-buffer call and the chunked-prefill call reject bad arguments
    before touching the device."""
    lib = _ffi.lib()
    p = ctypes.c_void_p(0x100000)
    ws = ctypes.c_void_p(0x200000)   # 256-byte aligned
    need = lib.bw_attn_fwd_host_workspace_size(1, 8, 2, 256, 128)
    a256 = lambda x: (x + 255) // 256 * 256
    assert need == 2 * a256(8 * 256 * 128 * 2) + 2 * a256(2 * 256 * 128 * 2) + a256(8 * 256 * 4)
    assert lib.bw_attn_fwd_host_workspace_size(0, 8, 2, 256, 128) == 0
    host = lambda **kw: lib.bw_attn_fwd_host(kw.get("q", p), p, p, p, None, 1, kw.get("hq", 8), 2, 256,
                                             kw.get("d", 128), 0.1, 1, kw.get("layout", _ffi.BW_LAYOUT_BSHD), 4,
                                             kw.get("ws", ws), kw.get("nbytes", need), None)
    assert host(q=None) == _ffi.BW_ERR_NULL
    assert host(ws=None) == _ffi.BW_ERR_NULL
    assert host(d=96) == _ffi.BW_ERR_SHAPE
    assert host(hq=7) == _ffi.BW_ERR_SHAPE
    assert host(layout=5) == _ffi.BW_ERR_SHAPE
    assert host(nbytes=need - 1) == _ffi.BW_ERR_WORKSPACE
    assert host(ws=ctypes.c_void_p(0x200010)) == _ffi.BW_ERR_ALIGN
    off = lambda q_offset, sq=128: lib.bw_gqa_causal_offset_fwd(p, p, p, p, None, 1, 8, 2, sq, 512, 4, 128, 0.1,
                                                                q_offset, None, None)
    assert off(-1) == _ffi.BW_ERR_SHAPE
    assert off(1 << 30) == _ffi.BW_ERR_SHAPE
    assert off(0, sq=0) == _ffi.BW_ERR_SHAPE


def test_prefill_kernel_option_values():
    lib = _ffi.lib()
    old = lib.bw_get_option(_ffi.BW_OPT_PREFILL_KERNEL)
    assert old == 0                                   # default kernel
    for v in (0, 4, 5):
        assert lib.bw_set_option(_ffi.BW_OPT_PREFILL_KERNEL, v) == 0
    for v in (-1, 1, 2, 3, 6):                        # kernels 1-3 were removed
        assert lib.bw_set_option(_ffi.BW_OPT_PREFILL_KERNEL, v) == _ffi.BW_ERR_SHAPE
    lib.bw_set_option(_ffi.BW_OPT_PREFILL_KERNEL, old)
    # the P-in-TMEM switch went with kernel 1
    assert lib.bw_set_option(_ffi.BW_OPT_P_IN_TMEM, 1) == _ffi.BW_ERR_SHAPE
