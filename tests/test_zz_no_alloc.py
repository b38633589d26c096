"""The allocation-free decode entry point, bw_gqa_decode_static.

It exists for callers that cannot allocate device memory (allocator hooks,
memory-pool callbacks, host runtimes that own no allocator): it keeps its
scratch in a fixed array inside the library instead of a caller workspace.
This test calls it through the C ABI twice in a row and checks each result
against the workspace-taking bw_gqa_decode on the same inputs and against the
fp64 oracle, within the parity tolerances the other tests use; after the first
call (which does the set-up) the device's free memory must not change.  The file name sorts last so that a run
stopping at the first failure has already run every other test; it also works
alone in a fresh process (the first call does the per-device set-up)."""
import ctypes
import math

import numpy as np
import pytest
import torch

from oracle import attention_oracle as orc
from tests._util import LSE_TOL, O_TOL, seeded_bf16

pytestmark = pytest.mark.gpu


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _case(seed, B, Hq, Hkv, D, maxlen):
    rng = np.random.default_rng(seed)
    lens = rng.integers(1, maxlen + 1, B).astype(np.int32)
    offs = np.concatenate([[0], np.cumsum(lens)[:-1]]).astype(np.int64)
    total = int(lens.sum())
    q = seeded_bf16((B, Hq, D), seed).cuda()
    k = seeded_bf16((total, Hkv, D), seed + 1).cuda()
    v = seeded_bf16((total, Hkv, D), seed + 2).cuda()
    return q, k, v, torch.from_numpy(lens).cuda(), torch.from_numpy(offs).cuda(), total


def test_static_scratch_decode_matches_workspace_decode():
    from blackwell_b200 import _ffi
    lib = _ffi.lib()
    assert lib.bw_gqa_decode_static_scratch_bytes() == 32 << 20
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for seed, (B, Hq, Hkv, D, maxlen, chunk) in [(1, (6, 32, 4, 128, 5000, 256)), (2, (3, 16, 2, 64, 900, 0))]:
        q, k, v, lens, offs, total = _case(seed, B, Hq, Hkv, D, maxlen)
        scale = 1 / math.sqrt(D)
        # reference result: the existing entry point with a caller workspace
        ws = torch.empty(lib.bw_gqa_decode_workspace_size(B, Hq, Hkv, D, total, chunk), dtype=torch.uint8,
                         device="cuda")
        o_ref = torch.empty(B, Hq, D, dtype=torch.bfloat16, device="cuda")
        l_ref = torch.empty(B, Hq, dtype=torch.float32, device="cuda")
        rc = lib.bw_gqa_decode(_ptr(q), _ptr(k), _ptr(v), _ptr(lens), _ptr(offs), _ptr(o_ref), _ptr(l_ref), B, Hq,
                               Hkv, D, total, scale, chunk, _ptr(ws), ws.numel(), stream)
        assert rc == 0
        assert lib.bw_stream_status(stream) == 0
        ro, rl = orc.decode_reference(q, k, v, lens.cpu().numpy(), offs.cpu().numpy(), scale)
        outs = [(torch.full((B, Hq, D), float("nan"), dtype=torch.bfloat16, device="cuda"),
                 torch.full((B, Hq), float("nan"), dtype=torch.float32, device="cuda")) for _ in range(2)]
        torch.cuda.synchronize()
        free_before = None
        for i, (o, lse) in enumerate(outs):  # two calls in a row share (and reuse) the static scratch
            rc = lib.bw_gqa_decode_static(_ptr(q), _ptr(k), _ptr(v), _ptr(lens), _ptr(offs), _ptr(o), _ptr(lse), B,
                                          Hq, Hkv, D, total, scale, chunk, stream)
            assert rc == 0
            assert lib.bw_stream_status(stream) == 0
            if i == 0:
                free_before = torch.cuda.mem_get_info()[0]
            else:
                assert torch.cuda.mem_get_info()[0] == free_before   # the call allocated nothing
            assert (o.float() - o_ref.float()).abs().max().item() <= O_TOL
            assert (lse - l_ref).abs().max().item() <= LSE_TOL
            assert np.abs(o.float().cpu().numpy() - ro).max() <= O_TOL
            assert np.abs(lse.cpu().numpy() - rl).max() <= LSE_TOL


def test_static_scratch_rejects_oversize():
    from blackwell_b200 import _ffi
    lib = _ffi.lib()
    p = ctypes.c_void_p(0x100000)
    # 64 sequences, 8 KV heads, 16M tokens in 64-token chunks needs far more than 32 MiB
    rc = lib.bw_gqa_decode_static(p, p, p, p, p, p, None, 64, 64, 8, 128, 1 << 24, 0.08, 64, None)
    assert rc == _ffi.BW_ERR_WORKSPACE
