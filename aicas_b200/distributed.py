"""Sequence-sharded (split-KV) decode across GPUs.

Rank r of N owns cache positions ``[r*L/N, (r+1)*L/N)`` of every (request, KV
head).  Each rank runs the decode kernel on its shard and produces a normalised
fp32 partial output ``[B, Hq, D]`` with its base-2 LSE ``[B, Hq]``; ONE NCCL
all-gather of the packed partials (N x (B*Hq*D + B*Hq) floats) brings every
partial to every rank, and the merge kernel combines them.  The reference has
no multi-GPU code at all; this is the exchange step of its long-context path.

Decode batches that do not need a shared cache shard by request with no
collective at all (each rank runs :func:`aicas_b200.gqa_decode_attention` on
its own requests).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import ops


def shard_bounds(length: int, world: int, rank: int) -> tuple[int, int]:
    """[start, end) of the cache positions rank `rank` owns (ceil-sized shards)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    step = -(-length // world)
    start = min(length, rank * step)
    return start, min(length, start + step)


def local_lengths(kv_lens: torch.Tensor, start: int, end: int) -> torch.Tensor:
    """Valid positions of each request inside the shard [start, end)."""
    return (kv_lens.to(torch.int64) - start).clamp(0, end - start).to(torch.int32)


def pack_partials(partial_o: torch.Tensor, partial_lse: torch.Tensor) -> torch.Tensor:
    """One flat fp32 buffer [B*Hq*D + B*Hq] per rank, so a single collective moves both."""
    return torch.cat([partial_o.reshape(-1), partial_lse.reshape(-1)])


def unpack_partials(gathered: torch.Tensor, world: int, batch: int, heads: int, head_dim: int):
    """Inverse of :func:`pack_partials` over the all-gathered buffer:
    returns ([world, B, Hq, D], [world, B, Hq])."""
    per = batch * heads * (head_dim + 1)
    if gathered.numel() != world * per:
        raise ValueError(f"gathered buffer has {gathered.numel()} floats, expected {world * per}")
    g = gathered.view(world, per)
    o = g[:, : batch * heads * head_dim].reshape(world, batch, heads, head_dim)
    lse = g[:, batch * heads * head_dim :].reshape(world, batch, heads)
    return o, lse


def gather_partials(partial_o: torch.Tensor, partial_lse: torch.Tensor, group=None):
    world = dist.get_world_size(group)
    packed = pack_partials(partial_o, partial_lse)
    gathered = torch.empty(world * packed.numel(), dtype=packed.dtype, device=packed.device)
    dist.all_gather_into_tensor(gathered, packed, group=group)
    B, H, D = partial_o.shape
    return unpack_partials(gathered, world, B, H, D)


def sharded_gqa_decode(
    query: torch.Tensor,
    key_shard: torch.Tensor,
    value_shard: torch.Tensor,
    *,
    sm_scale: float,
    num_key_value_groups: int,
    kv_lens_local: torch.Tensor | None = None,
    group=None,
) -> torch.Tensor:
    """Decode attention over a cache sharded along the sequence across the ranks
    of `group`: partial on the local shard, one all-gather, merge.  Every rank
    returns the full ``[B, Hq, 1, D]`` output."""
    po, lse = ops.gqa_decode_partial(query, key_shard, value_shard, sm_scale=sm_scale,
                                     num_key_value_groups=num_key_value_groups, kv_lens=kv_lens_local)
    all_o, all_lse = gather_partials(po, lse, group)
    return ops.merge_partials(all_o, all_lse, out_dtype=query.dtype)
