"""Sequence-sharded (split-KV) decode across real GPUs: each rank runs the
partial decode kernel on its shard of the cache, then the partials are
combined either by the one-kernel NVLink peer exchange + merge or by one NCCL
all-gather and the merge kernel; or the decode kernel itself exchanges and
merges (the fused path, whose middle call goes through the merge kernel on the
same buffers so the two share the epoch).  Checked on every rank against the fp64
oracle of the whole cache (tolerance: the north-star bf16 bar, max-abs 2e-2
and mean-abs 2e-3); the peer path runs three calls in a row so both parities
of its double-buffered slots, and their reuse, are exercised.

Runs only where the process sees two or more GPUs; ranks are spawned child
processes with a short process-group timeout.
"""
from __future__ import annotations

import datetime
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, path: str, cases, out_dir: str):
    import torch.distributed as dist

    from aicas_b200 import distributed as adist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    device = torch.device("cuda", rank)
    torch.cuda.set_device(device)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=device,
                            timeout=datetime.timedelta(seconds=60))
    exchange = None
    try:
        q0 = cases[0][0]
        if path in ("peer", "fused"):
            exchange = adist.PeerExchange(q0.shape[0], q0.shape[1], q0.shape[3], device)
        for i, (q, k, v, lens) in enumerate(cases):
            L = k.shape[2]
            s0, s1 = adist.shard_bounds(L, world, rank)
            qd = q.to(device)
            kd = k[:, :, s0:s1].contiguous().to(device)
            vd = v[:, :, s0:s1].contiguous().to(device)
            local = adist.local_lengths(lens, s0, s1).to(device)
            out = adist.sharded_gqa_decode(qd, kd, vd, sm_scale=q.shape[-1] ** -0.5, num_key_value_groups=2,
                                           kv_lens_local=local, exchange=exchange,
                                           fused=(path == "fused" and i != 1))
            torch.cuda.synchronize(device)
            np.save(os.path.join(out_dir, f"out{rank}_{i}.npy"), out.float().cpu().numpy())
        from aicas_b200 import _native

        np.save(os.path.join(out_dir, f"err{rank}.npy"), np.array([_native.device_error_flags()]))
        dist.barrier(device_ids=[rank])
    finally:
        if exchange is not None:
            exchange.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("path", ["peer", "fused", "nccl"])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_split_kv_decode_across_gpus(tmp_path, world, path):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp

    from oracle import attention as oa
    from tests.conftest import bf16_tolerance_check

    B, Hq, Hkv, L, D = 3, 16, 8, 12288, 128
    cases = []
    for seed, lens in ((11, [L, 7001, 1]), (12, [5000, L, 6145]), (13, [1, 2, 12000])):
        # full caches, caches ending in either rank's shard, a one-token cache
        g = torch.Generator().manual_seed(seed)
        q = torch.randn(B, Hq, 1, D, generator=g).to(torch.bfloat16)
        k = torch.randn(B, Hkv, L, D, generator=g).to(torch.bfloat16)
        v = torch.randn(B, Hkv, L, D, generator=g).to(torch.bfloat16)
        cases.append((q, k, v, torch.tensor(lens, dtype=torch.int32)))
    mp.start_processes(_worker, args=(world, _free_port(), path, cases, str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    for i, (q, k, v, lens) in enumerate(cases):
        ref = oa.decode_ragged(q.float().numpy(), k.float().numpy(), v.float().numpy(), lens.tolist(), D ** -0.5, 2)
        for r in range(world):
            bf16_tolerance_check(np.load(tmp_path / f"out{r}_{i}.npy"), ref)
    for r in range(world):
        assert int(np.load(tmp_path / f"err{r}.npy")[0]) == 0
