"""Multi-GPU execution: one process per GPU, torch.distributed for the plumbing.

* Full-sequence attention (prefill, MHA) shards by (batch x KV-head group):
  every query head of a group reads only that group's K/V, so the units are
  independent and no data crosses GPUs.  ``unit_range`` / ``local_units`` give a
  rank its contiguous share (the C ABI's ``bw_shard_plan``).
* Split-KV decode over sequences too long for one GPU splits every sequence's
  keys across the ranks (``split_sequences``).  Each rank runs the decode on its
  keys (``bw_gqa_decode_partial``: fp32 O normalised by its own sum plus LSE),
  the partials are all-gathered into local buffers over NCCL, and every rank
  merges them with the LSE-combine kernel (``decode_sequence_parallel``).  The
  merge reads only local memory; no kernel reads a peer's memory.
"""
from __future__ import annotations

from typing import Callable, Optional

import numpy as np
import torch
import torch.distributed as dist

from . import attention


def unit_range(units: int, world: int, rank: int):
    """[begin, end) of the rank's contiguous share of `units` work units."""
    return attention.shard_plan(units, world, rank)


def local_units(B: int, Hkv: int, world: int, rank: int):
    """The (b, kv_group) units of this rank, in order."""
    b0, b1 = unit_range(B * Hkv, world, rank)
    return [(u // Hkv, u % Hkv) for u in range(b0, b1)]


def split_sequences(kv_lens, world: int, rank: int):
    """Split every sequence's keys into `world` contiguous pieces (sizes differ by
    at most one token).  Returns (local_lens int32 [B], starts int64 [B]): this
    rank's token count of each sequence and its first token inside that sequence."""
    lens = np.asarray(kv_lens, dtype=np.int64)
    base, rem = lens // world, lens % world
    starts = rank * base + np.minimum(rank, rem)
    local = base + (rank < rem)
    return local.astype(np.int32), starts.astype(np.int64)


def _all_gather(t: torch.Tensor, group) -> torch.Tensor:
    world = dist.get_world_size(group)
    out = torch.empty((world,) + tuple(t.shape), dtype=t.dtype, device=t.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, t.contiguous(), group=group)
    else:
        dist.all_gather(list(out.unbind(0)), t.contiguous(), group=group)
    return out


def decode_sequence_parallel(q, k_local, v_local, local_lens, local_offsets, scale=None, chunk=0, group=None,
                             local_decode: Optional[Callable] = None, combine: Optional[Callable] = None):
    """Decode with every sequence's keys spread over the ranks of `group`.

    q: [B, Hq, D] (same on every rank); k_local / v_local: this rank's keys,
    [local_tokens, Hkv, D], sequence b at rows [local_offsets[b], + local_lens[b]).
    Returns (O, LSE) of the full sequences on every rank.

    One collective per step: the rank's partial O (fp32 [B, Hq, D]) and LSE
    (fp32 [B, Hq]) are written into ONE packed buffer (O, then LSE, padded to 16
    bytes: ``attention.packed_split_floats``) and a single all-gather brings
    every rank's buffer; ``bw_lse_combine_packed`` merges straight from the
    gathered [world, packed] tensor.  `local_decode` and `combine` default to the
    native kernels; tests substitute CPU checkers (``combine`` then receives
    strided [world, B, Hq, D] / [world, B, Hq] views of the gathered buffer)."""
    B, Hq, D = q.shape
    n_o = B * Hq * D
    buf = torch.empty(attention.packed_split_floats(B, Hq, D), dtype=torch.float32, device=q.device)
    o_view, lse_view = buf[:n_o].view(B, Hq, D), buf[n_o:n_o + B * Hq].view(B, Hq)
    if local_decode is None:
        attention.gqa_decode_partial(q, k_local, v_local, local_lens, local_offsets, scale=scale, chunk=chunk,
                                     out=o_view, lse=lse_view)
    else:
        o_part, lse_part = local_decode(q, k_local, v_local, local_lens, local_offsets, scale=scale, chunk=chunk)
        o_view.copy_(o_part)
        lse_view.copy_(lse_part)
    gathered = _all_gather(buf, group)
    if combine is None:
        return attention.lse_combine_packed(gathered, B, Hq, D)
    return combine(gathered[:, :n_o].view(-1, B, Hq, D), gathered[:, n_o:n_o + B * Hq].view(-1, B, Hq))
