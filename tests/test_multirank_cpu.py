"""Host logic of the sequence-sharded decode on world_size 2 (and 4) gloo ranks
on CPU: shard bounds, per-shard lengths, packing of the (out, LSE) partials into
one collective buffer, the all-gather, unpacking, and the merge, with the
oracle standing in for the per-shard kernel.  No GPU."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from aicas_b200 import distributed as adist


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, q, k, v, lens, out_dir: str):
    from oracle import attention as oa

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        L = k.shape[2]
        s0, s1 = adist.shard_bounds(L, world, rank)
        local = adist.local_lengths(torch.tensor(lens), s0, s1)
        B, Hq, D = q.shape[0], q.shape[1], q.shape[3]
        po = np.zeros((B, Hq, D))
        pl = np.full((B, Hq), -np.inf)
        for b in range(B):
            n = int(local[b])
            if n == 0:
                continue
            kk, vv = k[b : b + 1, :, s0 : s0 + n].numpy(), v[b : b + 1, :, s0 : s0 + n].numpy()
            po[b] = oa.sdpa(q[b : b + 1].numpy(), kk, vv, 0.1, False, 2)[0, :, 0]
            pl[b] = oa.lse_base2(q[b : b + 1].numpy(), kk, 0.1, 2)[0]
        packed = adist.pack_partials(torch.from_numpy(po).float(), torch.from_numpy(pl).float())
        gathered = [torch.empty_like(packed) for _ in range(world)]
        dist.all_gather(gathered, packed)
        all_o, all_lse = adist.unpack_partials(torch.cat(gathered), world, B, Hq, D)
        merged = oa.merge(all_o.double().numpy(), all_lse.double().numpy())
        np.save(os.path.join(out_dir, f"rank{rank}.npy"), merged)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_decode_merge_on_gloo(tmp_path, world):
    from oracle import attention as oa

    g = torch.Generator().manual_seed(world)
    B, Hq, Hkv, L, D = 3, 4, 2, 301, 32
    q = torch.randn(B, Hq, 1, D, generator=g)
    k = torch.randn(B, Hkv, L, D, generator=g)
    v = torch.randn(B, Hkv, L, D, generator=g)
    lens = [301, 40, 160]  # request 1 lives entirely on the first shard(s): empty shards elsewhere
    mp.start_processes(_worker, args=(world, _free_port(), q, k, v, lens, str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    ref = oa.decode_ragged(q.numpy(), k.numpy(), v.numpy(), lens, 0.1, 2)[:, :, 0]
    for r in range(world):
        np.testing.assert_allclose(np.load(tmp_path / f"rank{r}.npy"), ref, rtol=0, atol=1e-6)


def test_shard_bounds_cover_the_cache_once():
    for L in (1, 7, 131072, 131073):
        for world in (1, 2, 4, 8):
            spans = [adist.shard_bounds(L, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == L
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            assert all(e >= s for s, e in spans)


def test_local_lengths_clip_to_the_shard():
    lens = torch.tensor([0, 5, 100, 250])
    assert adist.local_lengths(lens, 0, 100).tolist() == [0, 5, 100, 100]
    assert adist.local_lengths(lens, 100, 200).tolist() == [0, 0, 0, 100]
    assert adist.local_lengths(lens, 200, 300).tolist() == [0, 0, 0, 50]


def test_unpack_rejects_a_wrong_buffer():
    with pytest.raises(ValueError):
        adist.unpack_partials(torch.zeros(11), 2, 1, 1, 4)
