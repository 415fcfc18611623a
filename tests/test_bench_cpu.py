"""Host side of bench.py (no GPU): the config-5 cache is defined chunk by chunk,
so every rank count sees the same whole cache (the sharded result is checked
against one whole-cache reference at every N), and the two arms print one
config."""
from __future__ import annotations

import torch

import bench


def test_cfg5_shards_tile_one_cache():
    whole_k, whole_v = bench.cfg5_shard(0, 20000, "cpu")
    assert whole_k.shape == (bench.CFG5_B, 8, 20000, 128) and whole_k.dtype == torch.bfloat16
    for bounds in ((0, 16384, 20000), (0, 5000, 16384, 16385, 20000)):
        parts = [bench.cfg5_shard(a, b, "cpu") for a, b in zip(bounds[:-1], bounds[1:])]
        assert torch.equal(torch.cat([p[0] for p in parts], 2), whole_k)
        assert torch.equal(torch.cat([p[1] for p in parts], 2), whole_v)


def test_both_arms_print_one_config():
    ours = bench.cfg2_config(4)
    assert ours == bench.cfg2_config(4) and ours["parallelism"].startswith("dp4")
    assert "graph" not in ours  # how each arm runs the step is reported beside the config


def test_layer_chunks_cover_every_layer_once():
    chunks = bench._layer_chunks(28)
    covered = [layer for a, b in chunks for layer in range(a, b)]
    assert covered == list(range(28))
