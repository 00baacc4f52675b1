"""Multi-GPU plumbing for view-sharded and tile-strip-sharded rendering.

The forward renderer has no data exchange inside a frame: every GPU holds a
full replica of the Gaussians and renders its own views (or its own band of
tile rows of one large frame). The only collective is one broadcast of the
scene arrays at session start (one NCCL broadcast of a packed buffer over
NVLink); there is no per-frame collective. One process per GPU, launched by
torchrun; the rendezvous uses 127.0.0.1.
"""

from __future__ import annotations

import datetime
import os
from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass(frozen=True)
class RankInfo:
    rank: int
    world_size: int
    local_rank: int

    @property
    def is_root(self) -> bool:
        return self.rank == 0


def rank_info() -> RankInfo:
    return RankInfo(int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
                    int(os.environ.get("LOCAL_RANK", "0")))


def init_process_group(backend: str = "nccl", timeout_s: float = 120.0) -> RankInfo:
    """Initialises torch.distributed from the torchrun environment (no-op for one rank)."""
    info = rank_info()
    if info.world_size > 1 and not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        kwargs = {}
        if backend == "nccl":
            torch.cuda.set_device(info.local_rank)
            kwargs["device_id"] = torch.device("cuda", info.local_rank)
        dist.init_process_group(backend=backend, timeout=datetime.timedelta(seconds=timeout_s), **kwargs)
    return info


def view_shard(num_views: int, rank: int, world_size: int) -> list[int]:
    """Views rendered by `rank`: round-robin, so consecutive orbit views spread evenly."""
    if world_size <= 0 or not 0 <= rank < world_size:
        raise ValueError("rank must lie in [0, world_size)")
    return list(range(rank, num_views, world_size))


def tile_strips(grid_y: int, world_size: int) -> list[tuple[int, int]]:
    """Contiguous tile-row bands [begin, end) per rank, sizes differing by at most one."""
    if world_size <= 0:
        raise ValueError("world_size must be positive")
    base, extra = divmod(grid_y, world_size)
    bands, start = [], 0
    for r in range(world_size):
        size = base + (1 if r < extra else 0)
        bands.append((start, start + size))
        start += size
    return bands


def broadcast_scene(arrays: dict[str, torch.Tensor] | None, src: int = 0,
                    device: torch.device | None = None) -> dict[str, torch.Tensor]:
    """Replicates float32 scene arrays from `src` to every rank.

    Metadata (names and shapes) travels first as a small object broadcast;
    the payload is packed into one contiguous buffer and sent with a single
    broadcast, then unpacked into views. With one rank the input is returned.
    """
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return dict(arrays or {})
    rank = dist.get_rank()
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend() == "nccl" \
            else torch.device("cpu")
    meta = [None]
    if rank == src:
        meta = [[(k, tuple(v.shape)) for k, v in arrays.items()]]
    dist.broadcast_object_list(meta, src=src)
    layout = meta[0]
    sizes = [int(torch.Size(shape).numel()) for _, shape in layout]
    total = sum(sizes)
    if rank == src:
        packed = torch.cat([arrays[k].reshape(-1).to(device, torch.float32) for k, _ in layout]) if total else \
            torch.empty(0, device=device)
    else:
        packed = torch.empty(total, dtype=torch.float32, device=device)
    dist.broadcast(packed, src=src)
    out, offset = {}, 0
    for (name, shape), size in zip(layout, sizes):
        out[name] = packed[offset:offset + size].view(shape)
        offset += size
    return out
