"""B200-native (sm_100a) GQA / MHA flash-attention forward and split-KV decode.

The compute path is the native library ``libbw_attn.so`` (hand-written
tcgen05 / TMA kernels behind a C ABI, ``include/bw_attn.h``).  This package is
the Python host side: a ctypes binding (``_ffi``) and torch-tensor wrappers
(``attention``) that mirror the reference's Python entry points.
"""
from .attention import (  # noqa: F401
    gqa_fwd, gqa_causal_fwd, gqa_split_fwd, gqa_causal_offset_fwd, mha_fwd, gqa_decode, gqa_decode_paged, gqa_decode_partial,
    lse_combine, qk_norm_rope, gqa_fused_fwd, sdpa_gqa, sdpa_gqa_causal, stream_status, set_option, get_option,
    shard_plan, decode_workspace_size, attention_from_host, host_workspace_size, mha_fwd_f32,
)
