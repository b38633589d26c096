"""Multi-process (world size 2 and 3, gloo, CPU) tests of the multi-GPU host logic:
the unit sharding and the sequence-parallel decode exchange (split keys ->
local partials -> all-gather -> LSE merge).  The per-rank compute is the CPU
oracle here; on GPUs the same code runs the native kernels over NCCL."""
import math
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from blackwell_b200 import distributed as bwd
from oracle import attention_oracle as orc


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _oracle_partial(q, k, v, lens, offs, scale=None, chunk=0):
    """CPU stand-in for bw_gqa_decode_partial: per-sequence partial over local keys,
    (0, -inf) for a sequence without local keys."""
    B, Hq, D = q.shape
    o = torch.zeros(B, Hq, D)
    l = torch.full((B, Hq), float("-inf"))
    lens = np.asarray(lens)
    nz = np.nonzero(lens)[0]
    if len(nz):
        ro, rl = orc.decode_reference(q[nz], k, v, lens[nz], np.asarray(offs)[nz], scale or 1 / math.sqrt(D))
        o[nz] = torch.from_numpy(ro)
        l[nz] = torch.from_numpy(rl)
    return o, l


def _oracle_combine(o_all, lse_all):
    o, l = orc.lse_combine_reference(o_all.numpy(), lse_all.numpy())
    return torch.from_numpy(o), torch.from_numpy(l)


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        # --- unit sharding covers every (b, group) exactly once
        units = bwd.local_units(3, 5, world, rank)
        gathered = [None] * world
        dist.all_gather_object(gathered, units)
        flat = [u for part in gathered for u in part]
        assert sorted(flat) == [(b, g) for b in range(3) for g in range(5)]

        # --- sequence-parallel decode
        rng = np.random.default_rng(0)
        B, Hq, Hkv, D = 4, 8, 2, 64
        lens = np.array([1, 2, 37, 301])
        offs = np.concatenate([[0], np.cumsum(lens)[:-1]])
        g = torch.Generator().manual_seed(7)
        qq = torch.randn(B, Hq, D, generator=g)
        k = torch.randn(int(lens.sum()), Hkv, D, generator=g)
        v = torch.randn(int(lens.sum()), Hkv, D, generator=g)
        loc_lens, starts = bwd.split_sequences(lens, world, rank)
        rows = np.concatenate([np.arange(offs[b] + starts[b], offs[b] + starts[b] + loc_lens[b]) for b in range(B)])
        k_loc, v_loc = k[rows], v[rows]
        loc_offs = np.concatenate([[0], np.cumsum(loc_lens)[:-1]]).astype(np.int64)
        o, l = bwd.decode_sequence_parallel(qq, k_loc, v_loc, loc_lens, loc_offs, local_decode=_oracle_partial,
                                            combine=_oracle_combine)
        ro, rl = orc.decode_reference(qq, k, v, lens, offs, 1 / math.sqrt(D))
        assert np.abs(o.numpy() - ro).max() < 1e-5
        assert np.abs(l.numpy() - rl).max() < 1e-5
        q.put((rank, "ok"))
    except Exception as e:  # report to the parent instead of hanging it
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_sharding_and_sequence_parallel_decode(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    assert results == {r: "ok" for r in range(world)}, results


def test_split_sequences_partitions():
    lens = [0, 1, 5, 1000, 3]
    for world in (1, 2, 3, 8):
        parts = [bwd.split_sequences(lens, world, r) for r in range(world)]
        tot = sum(p[0].astype(np.int64) for p in parts)
        np.testing.assert_array_equal(tot, lens)
        for b in range(len(lens)):  # contiguous, ordered pieces
            pos = 0
            for loc, st in parts:
                assert st[b] == pos
                pos += loc[b]
