"""Failure detection without a GPU fault: every device-side wait is bounded.
A test hook makes the producer withhold its first K tile; the consumers' waits
expire after the (short) configured bound, the kernel unwinds, and the call
reports BW_ERR_TIMEOUT.  The context stays usable for the next call."""
import math

import pytest
import torch

from tests._util import seeded_bf16

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("kernel,D", [(0, 64), (0, 128), (4, 128), (4, 64), (5, 64)],
                         ids=["auto_d64", "auto_d128", "k4_d128", "k4_d64", "k5_d64"])
def test_withheld_tile_reports_timeout_and_recovers(kernel, D):
    """Each prefill kernel at both head dimensions: the withheld K tile makes
    every role's bounded wait expire."""
    import blackwell_b200 as bw
    from blackwell_b200 import _ffi
    q = seeded_bf16((1, 2, 256, D), 1).cuda()
    k = seeded_bf16((1, 2, 256, D), 2).cuda()
    v = seeded_bf16((1, 2, 256, D), 3).cuda()
    old_t = bw.get_option(_ffi.BW_OPT_TIMEOUT_NS)
    old_k = bw.get_option(_ffi.BW_OPT_PREFILL_KERNEL)
    try:
        bw.set_option(_ffi.BW_OPT_PREFILL_KERNEL, kernel)
        bw.set_option(_ffi.BW_OPT_TIMEOUT_NS, 50_000_000)   # 50 ms
        bw.set_option(_ffi.BW_OPT_DEBUG_FLAGS, 1)
        bw.mha_fwd(q, k, v)
        assert bw.stream_status() == _ffi.BW_ERR_TIMEOUT
    finally:
        bw.set_option(_ffi.BW_OPT_DEBUG_FLAGS, 0)
        bw.set_option(_ffi.BW_OPT_TIMEOUT_NS, old_t)
        bw.set_option(_ffi.BW_OPT_PREFILL_KERNEL, old_k)
    assert bw.stream_status() == 0
    o, lse = bw.mha_fwd(q, k, v)
    assert bw.stream_status() == 0
    ref = torch.nn.functional.scaled_dot_product_attention(q.float(), k.float(), v.float())
    assert (o.float() - ref).abs().max().item() < 2e-2


def test_errors_are_per_stream():
    """A call whose waits time out (withheld K tile) on one stream and a normal
    call on another stream: each stream's status reports only its own call, and
    reading one does not clear the other."""
    import blackwell_b200 as bw
    from blackwell_b200 import _ffi
    q = seeded_bf16((1, 2, 256, 128), 4).cuda()
    k = seeded_bf16((1, 2, 256, 128), 5).cuda()
    v = seeded_bf16((1, 2, 256, 128), 6).cuda()
    s_bad, s_good = torch.cuda.Stream(), torch.cuda.Stream()
    torch.cuda.synchronize()
    old_t = bw.get_option(_ffi.BW_OPT_TIMEOUT_NS)
    try:
        bw.set_option(_ffi.BW_OPT_TIMEOUT_NS, 50_000_000)   # 50 ms
        bw.set_option(_ffi.BW_OPT_DEBUG_FLAGS, 1)            # read at launch: only the next call withholds
        with torch.cuda.stream(s_bad):
            bw.mha_fwd(q, k, v)
        bw.set_option(_ffi.BW_OPT_DEBUG_FLAGS, 0)
        with torch.cuda.stream(s_good):
            o, _ = bw.mha_fwd(q, k, v)
        with torch.cuda.stream(s_good):
            assert bw.stream_status() == _ffi.BW_OK
        with torch.cuda.stream(s_bad):
            assert bw.stream_status() == _ffi.BW_ERR_TIMEOUT
            assert bw.stream_status() == _ffi.BW_OK          # read and cleared
    finally:
        bw.set_option(_ffi.BW_OPT_DEBUG_FLAGS, 0)
        bw.set_option(_ffi.BW_OPT_TIMEOUT_NS, old_t)
    torch.cuda.synchronize()
    ref = torch.nn.functional.scaled_dot_product_attention(q.float(), k.float(), v.float())
    assert (o.float() - ref).abs().max().item() < 2e-2
