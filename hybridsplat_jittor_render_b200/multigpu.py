"""Multi-GPU plumbing for view-sharded and tile-strip-sharded rendering.

The forward renderer has no data exchange inside a frame: every GPU holds a
full replica of the Gaussians and renders its own views (or its own band of
tile rows of one large frame). The only collectives are at session start: one
NCCL broadcast of the scene arrays from the root rank straight into every
rank's device buffers (over NVLink), plus a few host values (per-rank timings,
a barrier). They go through the library's NCCL communicator
(hs_b200_comm_*_v1 in include/hybridsplat_b200_ext.h); this module only finds
the ranks and hands the 128-byte NCCL id from rank 0 to the others over a
plain TCP socket, so no deep-learning framework is needed. One process per
GPU (torchrun or any launcher that sets RANK / WORLD_SIZE / LOCAL_RANK /
MASTER_ADDR / MASTER_PORT); the rendezvous uses 127.0.0.1 by default.
"""

from __future__ import annotations

import ctypes
import os
import socket
import time
from dataclasses import dataclass
from typing import Any, Callable, Sequence

from .native_runtime import check_status, error_buffer, load_native_library

ID_BYTES = 128
_MAGIC = b"HSB2"


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


@dataclass(frozen=True)
class PackedLayout:
    """Layout of named float32 arrays packed into one flat buffer, each at a
    256-byte aligned offset (so 16-byte vector loads of any row stay aligned):
    the scene is uploaded and broadcast as one buffer and every rank takes the
    same views of it."""

    entries: tuple[tuple[str, tuple[int, ...], int], ...]  # name, shape, offset in float32 elements
    total: int                                             # float32 elements

    ALIGN = 64  # float32 elements = 256 bytes

    @classmethod
    def of(cls, shapes: Sequence[tuple[str, tuple[int, ...]]]) -> "PackedLayout":
        entries, offset = [], 0
        for name, shape in shapes:
            count = 1
            for d in shape:
                count *= int(d)
            entries.append((name, tuple(int(d) for d in shape), offset))
            offset += (count + cls.ALIGN - 1) // cls.ALIGN * cls.ALIGN
        return cls(tuple(entries), max(offset, cls.ALIGN))

    def pack(self, arrays: dict[str, Any], out: Any) -> None:
        """Copies host float32 arrays (numpy) into the flat host buffer `out`."""
        for name, shape, offset in self.entries:
            flat = arrays[name].reshape(-1)
            if tuple(arrays[name].shape) != shape:
                raise ValueError(f"{name}: shape {tuple(arrays[name].shape)} != {shape}")
            out[offset:offset + flat.shape[0]] = flat

    def views(self, flat: Any) -> dict[str, Any]:
        """Named views of a flat float32 buffer (any array type with slicing
        and reshape, e.g. a device tensor)."""
        out = {}
        for name, shape, offset in self.entries:
            count = 1
            for d in shape:
                count *= d
            out[name] = flat[offset:offset + count].reshape(shape)
        return out


def rendezvous_port() -> int:
    """TCP port of the id hand-over: HS_B200_RENDEZVOUS_PORT, else MASTER_PORT + 1."""
    if "HS_B200_RENDEZVOUS_PORT" in os.environ:
        return int(os.environ["HS_B200_RENDEZVOUS_PORT"])
    return int(os.environ.get("MASTER_PORT", "29500")) + 1


def rendezvous_unique_id(rank: int, world_size: int, make_id: Callable[[], bytes], *,
                         addr: str = "127.0.0.1", port: int | None = None, timeout_s: float = 120.0) -> bytes:
    """Hands rank 0's ID_BYTES-byte id to every rank.

    Rank 0 calls make_id(), listens on (addr, port) and sends the id to each
    of the other world_size - 1 ranks as they connect; the others connect
    (retrying until timeout_s) and receive it. A rank that does not show up
    within timeout_s makes rank 0 raise TimeoutError; a missing rank 0 makes
    the others raise TimeoutError.
    """
    if world_size <= 0 or not 0 <= rank < world_size:
        raise ValueError("rank must lie in [0, world_size)")
    port = rendezvous_port() if port is None else int(port)
    deadline = time.monotonic() + timeout_s
    if rank == 0:
        unique = bytes(make_id())
        if len(unique) != ID_BYTES:
            raise ValueError(f"make_id() returned {len(unique)} bytes, expected {ID_BYTES}")
        if world_size == 1:
            return unique
        with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as server:
            server.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEADDR, 1)
            server.bind((addr, port))
            server.listen(world_size)
            joined = 0
            while joined < world_size - 1:
                left = deadline - time.monotonic()
                if left <= 0:
                    raise TimeoutError(f"rendezvous: {joined} of {world_size - 1} ranks joined within {timeout_s} s")
                server.settimeout(left)
                try:
                    conn, _ = server.accept()
                except socket.timeout as exc:
                    raise TimeoutError(
                        f"rendezvous: {joined} of {world_size - 1} ranks joined within {timeout_s} s") from exc
                with conn:
                    conn.sendall(_MAGIC + unique)
                joined += 1
        return unique
    while True:
        try:
            with socket.create_connection((addr, port), timeout=max(0.1, deadline - time.monotonic())) as conn:
                data = b""
                while len(data) < len(_MAGIC) + ID_BYTES:
                    chunk = conn.recv(len(_MAGIC) + ID_BYTES - len(data))
                    if not chunk:
                        break
                    data += chunk
            if data[:len(_MAGIC)] == _MAGIC and len(data) == len(_MAGIC) + ID_BYTES:
                return data[len(_MAGIC):]
        except OSError:
            pass
        if time.monotonic() > deadline:
            raise TimeoutError(f"rendezvous: rank 0 at {addr}:{port} not reached within {timeout_s} s")
        time.sleep(0.1)


class Communicator:
    """NCCL communicator of one rank (hs_b200_comm_*_v1).

    All operations return or raise within timeout_s: a rank that never joins
    or leaves mid-operation raises NativeRasterizerError on the others.
    """

    def __init__(self, device: int, rank: int, world_size: int, unique_id: bytes, *, timeout_s: float = 120.0,
                 library: ctypes.CDLL | None = None):
        self._lib = library if library is not None else load_native_library()
        self.device, self.rank, self.world_size = int(device), int(rank), int(world_size)
        self._handle = ctypes.c_void_p()
        raw = (ctypes.c_uint8 * ID_BYTES).from_buffer_copy(bytes(unique_id))
        error = error_buffer()
        status = self._lib.hs_b200_comm_create_v1(self.device, self.world_size, self.rank, raw, float(timeout_s),
                                                   ctypes.byref(self._handle), error, len(error))
        check_status(status, "hs_b200_comm_create_v1", error)

    @staticmethod
    def new_unique_id(library: ctypes.CDLL | None = None) -> bytes:
        lib = library if library is not None else load_native_library()
        raw = (ctypes.c_uint8 * ID_BYTES)()
        error = error_buffer()
        check_status(lib.hs_b200_comm_unique_id_v1(raw, error, len(error)), "hs_b200_comm_unique_id_v1", error)
        return bytes(raw)

    @classmethod
    def from_env(cls, device: int | None = None, *, timeout_s: float = 120.0,
                 library: ctypes.CDLL | None = None) -> "Communicator":
        """Communicator of this process's rank from the launcher's environment."""
        info = rank_info()
        lib = library if library is not None else load_native_library()
        unique = rendezvous_unique_id(info.rank, info.world_size, lambda: cls.new_unique_id(lib),
                                      addr=os.environ.get("MASTER_ADDR", "127.0.0.1"), timeout_s=timeout_s)
        return cls(info.local_rank if device is None else device, info.rank, info.world_size, unique,
                   timeout_s=timeout_s, library=lib)

    @property
    def handle(self) -> ctypes.c_void_p:
        if not self._handle:
            raise RuntimeError("communicator is closed")
        return self._handle

    def broadcast(self, pointer: int, nbytes: int, *, root: int = 0, stream: int | None = None) -> None:
        """In-place broadcast of nbytes of device memory at `pointer` from `root`."""
        error = error_buffer()
        status = self._lib.hs_b200_comm_broadcast_v1(self.handle, ctypes.c_void_p(pointer), int(nbytes), int(root),
                                                     ctypes.c_void_p(stream or 0), error, len(error))
        check_status(status, "hs_b200_comm_broadcast_v1", error)

    def broadcast_buffer(self, buffer: Any, *, root: int = 0, stream: int | None = None) -> None:
        """Broadcast of a device array object exposing data_ptr(), numel() and element_size()."""
        self.broadcast(int(buffer.data_ptr()), int(buffer.numel()) * int(buffer.element_size()), root=root,
                       stream=stream)

    def allreduce_max(self, values: Sequence[float]) -> list[float]:
        n = len(values)
        src = (ctypes.c_double * n)(*[float(v) for v in values])
        dst = (ctypes.c_double * n)()
        error = error_buffer()
        status = self._lib.hs_b200_comm_allreduce_max_f64_v1(self.handle, src, dst, n, error, len(error))
        check_status(status, "hs_b200_comm_allreduce_max_f64_v1", error)
        return list(dst)

    def barrier(self) -> None:
        error = error_buffer()
        check_status(self._lib.hs_b200_comm_barrier_v1(self.handle, error, len(error)), "hs_b200_comm_barrier_v1",
                     error)

    def close(self) -> None:
        if self._handle:
            error = error_buffer()
            status = self._lib.hs_b200_comm_destroy_v1(self._handle, error, len(error))
            self._handle = ctypes.c_void_p()
            check_status(status, "hs_b200_comm_destroy_v1", error)

    def __enter__(self) -> "Communicator":
        return self

    def __exit__(self, *exc: Any) -> None:
        self.close()


class SoloCommunicator:
    """The single-rank stand-in of Communicator: no NCCL, every collective is
    the identity."""

    rank, world_size = 0, 1

    def broadcast(self, pointer: int, nbytes: int, *, root: int = 0, stream: int | None = None) -> None:
        return None

    def broadcast_buffer(self, buffer: Any, *, root: int = 0, stream: int | None = None) -> None:
        return None

    def allreduce_max(self, values: Sequence[float]) -> list[float]:
        return [float(v) for v in values]

    def barrier(self) -> None:
        return None

    def close(self) -> None:
        return None


def communicator(device: int | None = None, *, timeout_s: float = 120.0,
                 library: ctypes.CDLL | None = None) -> Communicator | SoloCommunicator:
    """Communicator of this process from the launcher's environment; a
    SoloCommunicator when WORLD_SIZE is 1."""
    if rank_info().world_size <= 1:
        return SoloCommunicator()
    return Communicator.from_env(device, timeout_s=timeout_s, library=library)
