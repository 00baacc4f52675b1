"""The library's NCCL communicator (hs_b200_comm_*_v1) on GPUs.

One rank on one GPU always; two ranks (two processes, one GPU each) when the
box has two GPUs: the id hand-over over TCP, an in-place broadcast of a packed
scene buffer straight into device memory, the max reduction of host values
and the barrier.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from hybridsplat_jittor_render_b200 import multigpu

pytestmark = pytest.mark.gpu


def test_single_rank_communicator():
    unique = multigpu.Communicator.new_unique_id()
    assert len(unique) == 128
    with multigpu.Communicator(0, 0, 1, unique, timeout_s=60) as comm:
        data = torch.arange(1000, dtype=torch.float32, device="cuda")
        comm.broadcast_buffer(data)
        torch.cuda.synchronize()
        assert torch.equal(data.cpu(), torch.arange(1000, dtype=torch.float32))
        assert comm.allreduce_max([3.0, -1.5]) == [3.0, -1.5]
        comm.barrier()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank: int, world: int, port: int, queue):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      HS_B200_RENDEZVOUS_PORT=str(port), NCCL_NVLS_ENABLE="0")
    try:
        torch.cuda.set_device(rank)
        comm = multigpu.communicator(timeout_s=60)
        layout = multigpu.PackedLayout.of([("xyz", (4097, 3)), ("rot", (4097, 4))])
        flat = torch.zeros(layout.total, dtype=torch.float32, device="cuda")
        if rank == 0:
            host = np.zeros(layout.total, np.float32)
            rng = np.random.default_rng(5)
            layout.pack({"xyz": rng.random((4097, 3), dtype=np.float32),
                         "rot": rng.random((4097, 4), dtype=np.float32)}, host)
            flat.copy_(torch.from_numpy(host))
        comm.broadcast_buffer(flat, stream=torch.cuda.current_stream().cuda_stream)
        views = layout.views(flat)
        checksum = float(sum(v.double().sum().item() for v in views.values()))
        peak = comm.allreduce_max([float(rank), 10.0 - rank])
        comm.barrier()
        comm.close()
        queue.put((rank, checksum, peak))
    except Exception as exc:  # pragma: no cover - reported to the parent
        queue.put((rank, repr(exc), None))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_ranks_broadcast_and_reduce():
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    results = sorted(queue.get(timeout=180) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert all(isinstance(r[1], float) for r in results), results
    assert results[0][1] == results[1][1]
    assert results[0][2] == results[1][2] == [1.0, 10.0]
