"""Multi-process host logic of the view / tile-strip sharded session, on CPU.

The per-frame path has no collective. At session start rank 0 hands its NCCL
id to the other ranks over TCP (multigpu.rendezvous_unique_id) and the scene
is packed into one buffer with a layout every rank derives by itself
(multigpu.PackedLayout) and broadcast once. Here two CPU processes run the
id hand-over and the packed broadcast (over gloo, standing in for the
library's NCCL broadcast, which needs GPUs), take their view shards, and a
rank that never joins makes the hand-over fail within its timeout.
"""

from __future__ import annotations

import os
import socket
import time

import numpy as np
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


def test_packed_layout_round_trip_and_alignment():
    rng = np.random.default_rng(0)
    arrays = {"xyz": rng.random((1001, 3), dtype=np.float32), "rot": rng.random((1001, 4), dtype=np.float32),
              "op": rng.random((1001, 1), dtype=np.float32)}
    layout = multigpu.PackedLayout.of([(k, v.shape) for k, v in arrays.items()])
    assert all(off % 64 == 0 for _, _, off in layout.entries)
    flat = np.zeros(layout.total, np.float32)
    layout.pack(arrays, flat)
    for name, view in layout.views(flat).items():
        assert np.array_equal(view, arrays[name])
    with pytest.raises(ValueError):
        layout.pack({"xyz": arrays["xyz"][:10], "rot": arrays["rot"], "op": arrays["op"]}, flat)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, id_port: int, queue):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    try:
        unique = multigpu.rendezvous_unique_id(rank, world, lambda: bytes(range(128)), port=id_port, timeout_s=60)
        dist.init_process_group("gloo", rank=rank, world_size=world, init_method=f"tcp://127.0.0.1:{port}")
        shapes = [("xyz", (1000, 3)), ("shs", (1000, 48)), ("opacity", (1000, 1))]
        layout = multigpu.PackedLayout.of(shapes)
        flat = torch.zeros(layout.total, dtype=torch.float32)
        if rank == 0:
            rng = np.random.default_rng(0)
            host = np.zeros(layout.total, np.float32)
            layout.pack({k: rng.random(s, dtype=np.float32) for k, s in shapes}, host)
            flat.copy_(torch.from_numpy(host))
        dist.broadcast(flat, src=0)
        replica = layout.views(flat)
        views = multigpu.view_shard(20, rank, world)
        checksum = float(sum(v.double().sum() for v in replica.values()))
        queue.put((rank, checksum, views, {k: tuple(v.shape) for k, v in replica.items()}, unique))
        dist.destroy_process_group()
    except Exception as exc:  # pragma: no cover - reported to the parent
        queue.put((rank, repr(exc), None, None, None))


def test_id_handover_packed_broadcast_and_shards_two_ranks():
    world, port, id_port = 2, _free_port(), _free_port()
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, id_port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = sorted(queue.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert all(isinstance(r[1], float) for r in results), results
    assert results[0][1] == results[1][1]
    assert results[0][3] == {"xyz": (1000, 3), "shs": (1000, 48), "opacity": (1000, 1)}
    assert sorted(results[0][2] + results[1][2]) == list(range(20))
    assert results[0][4] == results[1][4] == bytes(range(128))


def _lonely_root(id_port: int, queue):
    t0 = time.monotonic()
    try:
        multigpu.rendezvous_unique_id(0, 2, lambda: bytes(128), port=id_port, timeout_s=2.0)
        queue.put(("joined", time.monotonic() - t0))
    except TimeoutError as exc:
        queue.put((str(exc), time.monotonic() - t0))


def test_rank_that_never_joins_times_out():
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    proc = ctx.Process(target=_lonely_root, args=(_free_port(), queue))
    proc.start()
    message, elapsed = queue.get(timeout=60)
    proc.join(timeout=30)
    assert "0 of 1 ranks joined" in message
    assert elapsed < 10.0


def test_missing_root_times_out():
    t0 = time.monotonic()
    with pytest.raises(TimeoutError):
        multigpu.rendezvous_unique_id(1, 2, lambda: bytes(128), port=_free_port(), timeout_s=1.0)
    assert time.monotonic() - t0 < 10.0
