"""Multi-process host logic of the view/tile-strip sharding, on CPU with gloo.

Two ranks broadcast a scene once and take their view shards; nothing else is
exchanged (the per-frame path has no collective).
"""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from hybridsplat_jittor_render_b200 import multigpu


def test_view_shard_partition():
    for world in (1, 2, 3, 8):
        shards = [multigpu.view_shard(160, r, world) for r in range(world)]
        flat = sorted(v for s in shards for v in s)
        assert flat == list(range(160))
        assert max(map(len, shards)) - min(map(len, shards)) <= 1
    with pytest.raises(ValueError):
        multigpu.view_shard(10, 2, 2)


def test_tile_strips_cover_rows():
    for grid_y, world in ((53, 1), (53, 2), (135, 8), (3, 8)):
        bands = multigpu.tile_strips(grid_y, world)
        assert bands[0][0] == 0 and bands[-1][1] == grid_y
        assert all(a[1] == b[0] for a, b in zip(bands, bands[1:]))
        sizes = [e - b for b, e in bands]
        assert max(sizes) - min(sizes) <= 1


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, queue):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    try:
        info = multigpu.init_process_group("gloo", timeout_s=60)
        scene = None
        if info.is_root:
            g = torch.Generator().manual_seed(0)
            scene = {"xyz": torch.randn(1000, 3, generator=g), "shs": torch.randn(1000, 48, generator=g),
                     "opacity": torch.rand(1000, 1, generator=g)}
        replica = multigpu.broadcast_scene(scene, src=0, device=torch.device("cpu"))
        views = multigpu.view_shard(20, info.rank, info.world_size)
        checksum = float(sum(v.double().sum() for v in replica.values()))
        queue.put((rank, checksum, views, {k: tuple(v.shape) for k, v in replica.items()}))
        dist.destroy_process_group()
    except Exception as exc:  # pragma: no cover - reported to the parent
        queue.put((rank, repr(exc), None, None))


def test_broadcast_scene_and_shard_with_gloo():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = sorted(queue.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert all(isinstance(r[1], float) for r in results), results
    assert results[0][1] == results[1][1]
    assert results[0][3] == {"xyz": (1000, 3), "shs": (1000, 48), "opacity": (1000, 1)}
    assert sorted(results[0][2] + results[1][2]) == list(range(20))
