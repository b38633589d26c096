"""Sequence-parallel decode over NCCL on 2+ GPUs (skipped with fewer GPUs):
every rank holds a slice of each sequence's keys, runs the native partial
decode, all-gathers the partials into local buffers and merges them."""
import math
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    try:
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
        from blackwell_b200 import distributed as bwd
        from oracle import attention_oracle as orc
        B, Hq, Hkv, D = 4, 64, 8, 128
        lens = np.array([5, 1024, 3000, 9000])
        offs = np.concatenate([[0], np.cumsum(lens)[:-1]])
        g = torch.Generator().manual_seed(3)
        qq = torch.randn(B, Hq, D, generator=g).bfloat16()
        k = torch.randn(int(lens.sum()), Hkv, D, generator=g).bfloat16()
        v = torch.randn(int(lens.sum()), Hkv, D, generator=g).bfloat16()
        loc, st = bwd.split_sequences(lens, world, rank)
        rows = np.concatenate([np.arange(offs[b] + st[b], offs[b] + st[b] + loc[b]) for b in range(B)]).astype(np.int64)
        lo = np.concatenate([[0], np.cumsum(loc)[:-1]]).astype(np.int64)
        o, l = bwd.decode_sequence_parallel(qq.cuda(), k[rows].cuda().contiguous(), v[rows].cuda().contiguous(),
                                            torch.from_numpy(loc).cuda(), torch.from_numpy(lo).cuda())
        torch.cuda.synchronize()
        ro, rl = orc.decode_reference(qq.float(), k.float(), v.float(), lens, offs, 1 / math.sqrt(D))
        eo = float(np.abs(o.float().cpu().numpy() - ro).max())
        el = float(np.abs(l.cpu().numpy() - rl).max())
        q.put((rank, "ok" if eo <= 2e-2 and el <= 1e-3 else f"err {eo} {el}"))
        dist.destroy_process_group()
    except Exception as e:
        q.put((rank, repr(e)))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sequence_parallel_decode_nccl():
    import torch.multiprocessing as mp
    world = min(torch.cuda.device_count(), 4)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    assert results == {r: "ok" for r in range(world)}, results
