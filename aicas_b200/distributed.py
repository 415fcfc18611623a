"""Sequence-sharded (split-KV) decode across GPUs.

Rank r of N owns cache positions ``[r*L/N, (r+1)*L/N)`` of every (request, KV
head).  Each rank runs the decode kernel on its shard and produces a normalised
fp32 partial output ``[B, Hq, D]`` with its base-2 LSE ``[B, Hq]``; ONE NCCL
all-gather of the packed partials (N x (B*Hq*D + B*Hq) floats) brings every
partial to every rank, and the merge kernel combines them.  The reference has
no multi-GPU code at all; this is the exchange step of its long-context path.

Two exchange paths are provided.  :class:`PeerExchange` moves the partials
over NVLink peer memory inside ONE kernel that also merges them (each rank
stores its partial into every rank's CUDA-IPC-mapped buffer, publishes a
flag, waits for the others' flags and merges); the NCCL path
(:func:`gather_partials`) is the fallback-free alternative for process groups
whose GPUs cannot map each other's memory.

Decode batches that do not need a shared cache shard by request with no
collective at all (each rank runs :func:`aicas_b200.gqa_decode_attention` on
its own requests).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

import ctypes

from . import _native, ops


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


class PeerExchange:
    """Symmetric exchange buffers over CUDA IPC for one process group and one
    partial shape [batch, heads, head_dim].  Construction is collective (every
    rank allocates its buffer and the 64-byte IPC handles are all-gathered);
    so is every :meth:`merge` call and :meth:`close`.  At most
    ``_native.MAX_EXCHANGE_RANKS`` ranks, one GPU each, all able to map each
    other's memory (NVLink / NVSwitch peers)."""

    def __init__(self, batch: int, heads: int, head_dim: int, device: torch.device, group=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > _native.MAX_EXCHANGE_RANKS:
            raise ValueError(f"peer exchange supports at most {_native.MAX_EXCHANGE_RANKS} ranks")
        self.shape = (batch, heads, head_dim)
        self.device = torch.device(device)
        lib = _native.lib()
        nbytes = lib.aicas_exchange_buffer_bytes(self.world, batch, heads, head_dim)
        if nbytes == 0:
            raise ValueError(f"bad exchange shape {self.shape} for {self.world} ranks")
        with torch.cuda.device(self.device):
            own = ctypes.c_void_p()
            handle = (ctypes.c_uint8 * _native.IPC_HANDLE_BYTES)()
            _native.check(lib.aicas_peer_buffer_alloc(nbytes, ctypes.byref(own), handle), "aicas_peer_buffer_alloc")
            self._own = own.value
            mine = torch.tensor(list(bytes(handle)), dtype=torch.uint8, device=self.device)
            every = torch.empty(self.world * _native.IPC_HANDLE_BYTES, dtype=torch.uint8, device=self.device)
            dist.all_gather_into_tensor(every, mine, group=group)
            handles = every.view(self.world, _native.IPC_HANDLE_BYTES).cpu()
            self._opened: list[int] = []
            peers: list[int] = []
            for r in range(self.world):
                if r == self.rank:
                    peers.append(self._own)
                    continue
                raw = (ctypes.c_uint8 * _native.IPC_HANDLE_BYTES)(*handles[r].tolist())
                ptr = ctypes.c_void_p()
                _native.check(lib.aicas_peer_buffer_open(raw, ctypes.byref(ptr)), "aicas_peer_buffer_open")
                self._opened.append(ptr.value)
                peers.append(ptr.value)
        self._peers = peers
        self._group = _native.PeerGroup()
        for r, ptr in enumerate(peers):
            self._group.peers[r] = ptr
        self._group.world, self._group.rank = self.world, self.rank
        dist.barrier(group=group)

    def decode(self, query: torch.Tensor, key_shard: torch.Tensor, value_shard: torch.Tensor, *, sm_scale: float,
               num_key_value_groups: int, kv_lens_local: torch.Tensor | None = None) -> torch.Tensor:
        """The sharded decode with the exchange fused into the decode kernel
        (one launch per rank, no partials in HBM): every rank returns the merged
        ``[B, Hq, 1, D]`` output.  Collective, like :meth:`merge`, and shares its
        buffers."""
        B, H, D = self.shape
        if query.shape[0] != B or query.shape[1] != H or query.shape[-1] != D:
            raise ValueError(f"query {tuple(query.shape)} does not match the exchange shape {self.shape}")
        if self._own is None:
            raise ValueError("the exchange is closed")
        return ops.gqa_decode_exchange(query, key_shard, value_shard, self._group, sm_scale=sm_scale,
                                       num_key_value_groups=num_key_value_groups, kv_lens=kv_lens_local)

    def merge(self, partial_o: torch.Tensor, partial_lse: torch.Tensor, out_dtype: torch.dtype) -> torch.Tensor:
        """All ranks' partials merged into a new ``[B, H, 1, D]`` tensor (every rank gets the full result)."""
        B, H, D = self.shape
        if tuple(partial_o.shape) != (B, H, D) or tuple(partial_lse.shape) != (B, H):
            raise ValueError(f"partials {tuple(partial_o.shape)} / {tuple(partial_lse.shape)} do not match {self.shape}")
        if partial_o.dtype != torch.float32 or partial_lse.dtype != torch.float32:
            raise ValueError("partials must be fp32")
        po = partial_o.contiguous()
        pl = partial_lse.contiguous()
        out = torch.empty(B, H, 1, D, dtype=out_dtype, device=po.device)
        p = _native.ExchangeParams()
        for r, ptr in enumerate(self._peers):
            p.peers[r] = ptr
        p.partial_o, p.partial_lse, p.out, p.lse = po.data_ptr(), pl.data_ptr(), out.data_ptr(), None
        p.o_stride_b, p.o_stride_h = out.stride(0), out.stride(1)
        p.world, p.rank, p.batch, p.num_heads, p.head_dim = self.world, self.rank, B, H, D
        if out_dtype not in ops._DTYPE_CODES:
            raise ValueError(f"unsupported output dtype {out_dtype}")
        p.dtype = ops._DTYPE_CODES[out_dtype]
        stream = torch.cuda.current_stream(po.device).cuda_stream
        _native.check(_native.lib().aicas_exchange_merge(ctypes.byref(p), stream), "aicas_exchange_merge")
        return out

    def close(self) -> None:
        """Collective: unmaps the peers' buffers and frees this rank's."""
        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        lib = _native.lib()
        for ptr in self._opened:
            lib.aicas_peer_buffer_close(ptr)
        dist.barrier(group=self.group)
        lib.aicas_peer_buffer_free(self._own)
        self._own = None
        self._opened = []


def sharded_gqa_decode(
    query: torch.Tensor,
    key_shard: torch.Tensor,
    value_shard: torch.Tensor,
    *,
    sm_scale: float,
    num_key_value_groups: int,
    kv_lens_local: torch.Tensor | None = None,
    group=None,
    exchange: PeerExchange | None = None,
    fused: bool = False,
) -> torch.Tensor:
    """Decode attention over a cache sharded along the sequence across the ranks
    of `group`: partial on the local shard, then either the one-kernel peer
    exchange + merge (`exchange` given) or one NCCL all-gather and the merge
    kernel.  With `exchange` and `fused`, the decode kernel itself exchanges and
    merges (:meth:`PeerExchange.decode`).  Every rank returns the full
    ``[B, Hq, 1, D]`` output."""
    if fused:
        if exchange is None:
            raise ValueError("the fused exchange needs a PeerExchange")
        return exchange.decode(query, key_shard, value_shard, sm_scale=sm_scale,
                               num_key_value_groups=num_key_value_groups, kv_lens_local=kv_lens_local)
    po, lse = ops.gqa_decode_partial(query, key_shard, value_shard, sm_scale=sm_scale,
                                     num_key_value_groups=num_key_value_groups, kv_lens=kv_lens_local)
    if exchange is not None:
        return exchange.merge(po, lse, query.dtype)
    all_o, all_lse = gather_partials(po, lse, group)
    return ops.merge_partials(all_o, all_lse, out_dtype=query.dtype)
