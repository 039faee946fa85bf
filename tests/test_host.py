"""Host-side logic on CPU: layer partitioning across ranks (with a world-size
2 gloo group for the y all-gather) and the MLX bridge's conversions."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from alloy_b200 import sharding


@pytest.mark.parametrize("H,G,world", [(128, 8, 1), (128, 8, 2), (128, 8, 4), (128, 8, 8),
                                       (64, 1, 2), (64, 1, 8), (8, 2, 4)])
def test_head_shards_cover_every_head_once(H, G, world):
    seen = []
    for r in range(world):
        s = sharding.head_shard(H, G, world, r)
        seen.extend(range(s.head_begin, s.head_begin + s.head_count))
        hpg = H // G
        assert s.group_begin == s.head_begin // hpg
        assert s.group_begin + s.group_count - 1 == (s.head_begin + s.head_count - 1) // hpg
        if G % world == 0:   # whole groups per rank: B/C columns are not shared
            assert s.head_begin % hpg == 0 and s.head_count % hpg == 0
    assert seen == list(range(H))


def test_head_shard_rejects_uneven_split():
    with pytest.raises(ValueError):
        sharding.head_shard(12, 4, 8, 0)


def test_batch_shards_cover_the_batch():
    for B, world in ((256, 8), (7, 3), (2, 4)):
        rows = []
        for r in range(world):
            b0, n = sharding.batch_shard(B, world, r)
            rows.extend(range(b0, b0 + n))
        assert rows == list(range(B))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gather_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        B, L, H, P = 2, 5, 8, 3
        full = torch.arange(B * L * H * P, dtype=torch.float32).reshape(B, L, H, P)
        s = sharding.head_shard(H, 2, world, rank)
        y_local = full[:, :, s.head_begin:s.head_begin + s.head_count].clone()
        y = sharding.allgather_heads(y_local, world)
        q.put((rank, bool(torch.equal(y, full))))
    finally:
        dist.destroy_process_group()


def test_allgather_heads_gloo_world2():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    results = dict(q.get(timeout=10) for _ in procs)
    assert results == {0: True, 1: True}


# ------------------------------------------------------------------ MLX bridge
def test_bridge_numpy_round_trip_on_cpu():
    from alloy_b200 import mlx_bridge
    a = np.arange(12, dtype=np.float32).reshape(3, 4)
    t = mlx_bridge.to_torch(a, device="cpu")
    assert t.dtype == torch.float32 and np.array_equal(t.numpy(), a)
    t16 = mlx_bridge.to_torch(a, device="cpu", dtype=torch.bfloat16)
    assert t16.dtype == torch.bfloat16


def test_patch_mamba_block_swaps_and_restores_methods():
    from alloy_b200 import mlx_bridge

    class FakeBlock:
        def _depthwise_conv1d(self, x_padded, L):
            return "ref"

        def _scan_chunk(self, *a, **k):
            return "ref"

        def _selective_scan(self, *a, **k):
            return "ref"

        def _selective_scan_sequential(self, *a, **k):
            return "ref"

    saved = mlx_bridge.patch_mamba_block(FakeBlock, device="cpu")
    assert FakeBlock._selective_scan is not saved["_selective_scan"]
    for name, fn in saved.items():
        setattr(FakeBlock, name, fn)
    assert FakeBlock()._selective_scan() == "ref"


def test_streamed_prefill_rejects_unpinned_or_device_activations():
    from alloy_b200 import mixer
    x = torch.zeros((1, 8, 288), dtype=torch.bfloat16)
    dt = torch.zeros((1, 8, 8), dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="pinned"):
        mixer.ssd_combined_streamed(x, dt, None, None, None, None, None, n_heads=8,
                                    head_dim=32, d_state=16, n_groups=1)
    with pytest.raises(ValueError, match="CPU tensor"):
        mixer.ssd_combined_streamed(None, dt, None, None, None, None, None, n_heads=8,
                                    head_dim=32, d_state=16, n_groups=1)
