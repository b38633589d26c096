"""ctypes binding of libbw_attn.so (the C ABI declared in include/bw_attn.h).

Loading fails loudly: there is no fallback implementation anywhere in this
package.  Build the library with ``python -m blackwell_b200.build``.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libbw_attn.so"

BW_OK, BW_ERR_SHAPE, BW_ERR_ALIGN, BW_ERR_CUDA, BW_ERR_TIMEOUT, BW_ERR_NCCL, BW_ERR_NULL, BW_ERR_WORKSPACE = range(8)
BW_LAYOUT_BHSD, BW_LAYOUT_BSHD = 0, 1
BW_OPT_TIMEOUT_NS, BW_OPT_P_IN_TMEM, BW_OPT_DEBUG_FLAGS, BW_OPT_MAX_CTAS, BW_OPT_EXP_POLY, BW_OPT_PREFILL_KERNEL = 1, 2, 3, 4, 5, 6

# Every symbol the header declares, with (restype, argtypes).
_vp, _i, _i64, _f, _sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_size_t


class BwStrides(ctypes.Structure):
    _fields_ = [("q", ctypes.c_int64 * 3), ("k", ctypes.c_int64 * 3), ("v", ctypes.c_int64 * 3),
                ("o", ctypes.c_int64 * 3)]


_SP = ctypes.POINTER(BwStrides)
SIGNATURES = {
    "bw_gqa_fwd": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _f, _SP, _vp]),
    "bw_gqa_causal_fwd": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _f, _SP, _vp]),
    "bw_gqa_split_fwd": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _f, _i, _SP, _vp]),
    "bw_mha_fwd": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _f, _SP, _vp]),
    "bw_mha_f32_workspace_size": (_sz, [_i, _i, _i, _i]),
    "bw_mha_fwd_f32": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _f, _SP, _vp, _sz, _vp]),
    "bw_gqa_decode_workspace_size": (_sz, [_i, _i, _i, _i, _i64, _i]),
    "bw_gqa_decode": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i64, _f, _i, _vp, _sz, _vp]),
    "bw_gqa_decode_paged": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _f, _i, _vp, _sz,
                                 _vp]),
    "bw_gqa_decode_partial": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i64, _f, _i, _vp, _sz, _vp]),
    "bw_gqa_decode_static_scratch_bytes": (_sz, []),
    "bw_gqa_decode_static": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i64, _f, _i, _vp]),
    "bw_lse_combine": (_i, [_vp, _vp, _i, _i, _i, _i, _vp, _vp, _vp]),
    "bw_decode_packed_split_floats": (_sz, [_i, _i, _i]),
    "bw_lse_combine_packed": (_i, [_vp, _i, _i, _i, _i, _vp, _vp, _vp]),
    "bw_qk_norm_rope": (_i, [_vp, _vp, _i, _i, _i, _i, _vp, _vp, _vp, _i, _i, _vp, _f, _i, _vp, _vp]),
    "bw_gqa_fused_workspace_size": (_sz, [_i, _i, _i, _i, _i]),
    "bw_gqa_causal_offset_fwd": (_i, [_vp] * 5 + [_i] * 7 + [_f, _i, _vp, _vp]),
    "bw_attn_fwd_host_workspace_size": (_sz, [_i, _i, _i, _i, _i]),
    "bw_attn_fwd_host": (_i, [_vp] * 5 + [_i] * 5 + [_f, _i, _i, _i, _vp, _sz, _vp]),
    "bw_gqa_fused_fwd": (_i, [_vp] * 10 + [_i] * 8 + [_f, _i, _f, _i, _vp, _sz, _vp]),
    "bw_stream_status": (_i, [_vp]),
    "bw_set_option": (_i, [_i, _i64]),
    "bw_get_option": (_i64, [_i]),
    "bw_shard_plan": (_i, [_i64, _i, _i, ctypes.POINTER(_i64), ctypes.POINTER(_i64)]),
    "bw_strerror": (ctypes.c_char_p, [_i]),
    "bw_version": (ctypes.c_char_p, []),
}

_lib = None
_lock = threading.Lock()


class BwError(RuntimeError):
    def __init__(self, code: int, where: str):
        self.code = code
        super().__init__(f"{where}: {strerror(code)} (code {code})")


def lib() -> ctypes.CDLL:
    """The loaded native library (raises if it was not built)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not LIB_PATH.exists():
                    raise RuntimeError(f"native library missing: {LIB_PATH} "
                                       "(build it with `python -m blackwell_b200.build`)")
                handle = ctypes.CDLL(str(LIB_PATH))
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(handle, name)
                    fn.restype, fn.argtypes = res, args
                _lib = handle
    return _lib


def strerror(code: int) -> str:
    return lib().bw_strerror(code).decode()


def check(code: int, where: str) -> None:
    if code != BW_OK:
        raise BwError(code, where)
