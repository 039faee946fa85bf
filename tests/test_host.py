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


def _torch_scan(x, B, C, h0, la, want_state, reverse=False):
    """The per-step recurrence h_t = exp(la_t) h_{t-1} + B_t x_t^T, y_t = C_t h_t
    (alloy/models/mamba_block.py:160-204), float64 on the CPU; ``reverse``
    walks the steps from the last."""
    if reverse:
        y, h = _torch_scan(x.flip(1), B.flip(1), C.flip(1), h0, la.flip(1), want_state)
        return y.flip(1), h
    b, L, H, _ = x.shape
    G = B.shape[2]
    Bh, Ch = B.repeat_interleave(H // G, 2), C.repeat_interleave(H // G, 2)
    h = torch.zeros(b, H, B.shape[3], x.shape[3], dtype=x.dtype) if h0 is None else h0.clone()
    ys = []
    for t in range(L):
        h = torch.exp(la[:, t])[:, :, None, None] * h + Bh[:, t, :, :, None] * x[:, t, :, None, :]
        ys.append((Ch[:, t, :, :, None] * h).sum(2))
    return torch.stack(ys, 1), (h if want_state else None)


@pytest.mark.parametrize("with_state", [False, True])
def test_scan_gradient_algebra_matches_autograd(with_state):
    # the decomposition selective_scan_backward runs on the GPU (three
    # rearranged scans and a reverse cumulative sum), here over a float64 scan
    from alloy_b200 import mixer
    g = torch.Generator().manual_seed(3)
    b, L, H, P, N, G = 2, 23, 4, 5, 3, 2
    r = lambda *s: torch.randn(*s, generator=g, dtype=torch.float64)
    x, B, C = r(b, L, H, P), r(b, L, G, N), r(b, L, G, N)
    la = -torch.rand(b, L, H, generator=g, dtype=torch.float64)
    h0 = r(b, H, N, P) if with_state else None
    U, V = r(b, L, H, P), r(b, H, N, P)
    leaves = [t.clone().requires_grad_() for t in (x, B, C, la)] + (
        [h0.clone().requires_grad_()] if with_state else [])
    y, hT = _torch_scan(leaves[0], leaves[1], leaves[2], leaves[4] if with_state else None,
                        leaves[3], True, False)
    ((y * U).sum() + (hT * V).sum()).backward()
    dx, dla, dB, dC, dh0 = mixer._scan_backward(_torch_scan, x, la, B, C, U, h0, V, "cpu")
    got = [dx, dB, dC, dla] + ([dh0] if with_state else [])
    want = [leaves[0].grad, leaves[1].grad, leaves[2].grad, leaves[3].grad] + (
        [leaves[4].grad] if with_state else [])
    for gt, wt in zip(got, want):
        assert torch.allclose(gt, wt, rtol=1e-9, atol=1e-9), (gt - wt).abs().max()
