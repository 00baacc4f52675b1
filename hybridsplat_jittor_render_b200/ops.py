"""Tensor-level operators over the C ABI (the Jittor op layer's counterpart).

Names, argument order and validation follow the reference operators:
``flashgs_forward`` (jittor_hybridsplat/ops/flashgs.py:54-136),
``rasterize_forward`` (ops/rasterizer.py:40-97) and the precise_* helpers
(ops/precise_*.py). Inputs are contiguous float32 CUDA ``torch.Tensor``s on
the context's device; outputs are newly allocated tensors with the
reference's shapes. Every call goes to the native library; there is no
fallback implementation.
"""

from __future__ import annotations

import ctypes
import math
from collections.abc import Sequence
from typing import Any, NamedTuple

import numpy as np
import torch

from . import native_runtime
from .native_runtime import (
    NativeRendererContext,
    check_status,
    error_buffer,
    load_native_library,
)


class FlashgsOutputs(NamedTuple):
    color: torch.Tensor
    other: torch.Tensor
    depth: torch.Tensor
    alpha: torch.Tensor
    normal: torch.Tensor
    median_depth: torch.Tensor
    distortion: torch.Tensor
    rendered: torch.Tensor


class RasterizerOutputs(NamedTuple):
    color: torch.Tensor
    auxiliary: torch.Tensor
    weight: torch.Tensor
    radii: torch.Tensor
    rendered: torch.Tensor


class TraceOutputs(NamedTuple):
    """Outputs of trace_reflection, named as the reference's OptixTraceOutputs
    fields (ops/optix.py)."""
    rgb: torch.Tensor
    depth: torch.Tensor
    acc: torch.Tensor
    normal: torch.Tensor
    dist: torch.Tensor
    aux: torch.Tensor
    mid: torch.Tensor
    wet: torch.Tensor


def _check_tensor(name: str, value: torch.Tensor, shape: tuple[int, ...], dtype=torch.float32) -> None:
    if not isinstance(value, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if tuple(value.shape) != shape:
        raise ValueError(f"{name} must have shape {shape}, got {tuple(value.shape)}")
    if value.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {value.dtype}")
    if not value.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def _finite(name: str, value: float, *, positive: bool = False) -> float:
    if isinstance(value, bool) or not isinstance(value, (int, float)):
        raise TypeError(f"{name} must be a CPU real scalar")
    result = float(value)
    if not math.isfinite(result) or (positive and result <= 0.0):
        raise ValueError(f"{name} must be {'finite and positive' if positive else 'finite'}")
    return result


def _vector(name: str, value: Sequence[float], count: int) -> tuple[float, ...]:
    if isinstance(value, torch.Tensor):
        value = value.detach().reshape(-1).cpu().tolist()
    flat: list[Any] = []
    for item in value:
        if isinstance(item, Sequence) and not isinstance(item, (str, bytes)):
            flat.extend(item)
        else:
            flat.append(item)
    if len(flat) != count:
        raise ValueError(f"{name} must contain {count} values")
    return tuple(_finite(f"{name}[{i}]", v) for i, v in enumerate(flat))


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


# Argument names of hs_flashgs_forward_f32_v1 after the handle, in ABI order
# (also the field names of HsB200FlashgsCallV2).
_FLASHGS_ORDER = (
    "point_count", "width", "height", "positions3", "shs48", "colors3", "use_sh", "opacities1",
    "covariance6", "scales2", "scale_modifier", "rotations4", "specular1", "roughness1",
    "camera_position3", "camera_rotation9", "focal_x", "focal_y", "z_far", "z_near", "background3",
    "initial_pair_capacity", "output_color3", "output_other2", "output_depth1", "output_alpha1",
    "output_normal3", "output_median_depth1", "output_distortion1", "output_num_rendered",
)
# The same for hs_rasterizer_forward_f32_v1 (fields of HsB200RasterizerCallV2).
_RASTERIZER_ORDER = (
    "point_count", "background5", "width", "height", "means3d", "colors5", "opacities", "scales2",
    "scale_modifier", "rotations4", "viewmatrix4x4", "projmatrix4x4", "camera_position3", "tan_fovx",
    "tan_fovy", "prefiltered", "output_color5", "output_aux7", "output_weight", "output_radii",
    "output_rendered",
)


def _flashgs_arguments(
    positions: torch.Tensor,
    shs: torch.Tensor,
    colors: torch.Tensor,
    opacities: torch.Tensor,
    covariance: torch.Tensor,
    scales: torch.Tensor,
    rotations: torch.Tensor,
    specular: torch.Tensor,
    roughness: torch.Tensor,
    *,
    width: int,
    height: int,
    use_sh: bool,
    camera_position: Sequence[float],
    camera_rotation: Sequence[float],
    focal_x: float,
    focal_y: float,
    z_far: float = 100.0,
    z_near: float = 0.01,
    background: Sequence[float] = (0.0, 0.0, 0.0),
    scale_modifier: float = 1.0,
    initial_pair_capacity: int = 1 << 20,
    out: FlashgsOutputs | None = None,
) -> tuple[dict[str, Any], FlashgsOutputs, list[Any]]:
    """Checks one FlashGS call; returns its named ABI arguments, the outputs
    and the host arrays that must outlive the call."""
    if isinstance(width, bool) or not isinstance(width, int) or width <= 0:
        raise ValueError("width must be a positive CPU integer")
    if isinstance(height, bool) or not isinstance(height, int) or height <= 0:
        raise ValueError("height must be a positive CPU integer")
    if not isinstance(use_sh, bool):
        raise TypeError("use_sh must be bool")
    if isinstance(initial_pair_capacity, bool) or not isinstance(initial_pair_capacity, int) or initial_pair_capacity <= 0:
        raise ValueError("initial_pair_capacity must be a positive CPU integer")
    count = int(positions.shape[0])
    for name, value, shape in (
        ("positions", positions, (count, 3)),
        ("shs", shs, (count, 48)),
        ("colors", colors, (count, 3)),
        ("opacities", opacities, (count, 1)),
        ("covariance", covariance, (count, 6)),
        ("scales", scales, (count, 2)),
        ("rotations", rotations, (count, 4)),
        ("specular", specular, (count, 1)),
        ("roughness", roughness, (count, 1)),
    ):
        _check_tensor(name, value, shape)
    position = _vector("camera_position", camera_position, 3)
    rotation = _vector("camera_rotation", camera_rotation, 9)
    bg = _vector("background", background, 3)
    scale = _finite("scale_modifier", scale_modifier, positive=True)
    fx = _finite("focal_x", focal_x, positive=True)
    fy = _finite("focal_y", focal_y, positive=True)
    far = _finite("z_far", z_far, positive=True)
    near = _finite("z_near", z_near, positive=True)
    if far <= near:
        raise ValueError("z_far must be greater than z_near")
    device = positions.device
    if out is None:
        f = dict(dtype=torch.float32, device=device)
        out = FlashgsOutputs(
            torch.empty((3, height, width), **f),
            torch.empty((2, height, width), **f),
            torch.empty((1, height, width), **f),
            torch.empty((1, height, width), **f),
            torch.empty((3, height, width), **f),
            torch.empty((1, height, width), **f),
            torch.empty((1, height, width), **f),
            torch.empty((1,), dtype=torch.int32, device=device),
        )
    position_host = (ctypes.c_float * 3)(*position)
    rotation_host = (ctypes.c_float * 9)(*rotation)
    bg_host = (ctypes.c_float * 3)(*bg)
    values = [count, width, height, _ptr(positions), _ptr(shs), _ptr(colors), int(use_sh), _ptr(opacities),
              _ptr(covariance), _ptr(scales), scale, _ptr(rotations), _ptr(specular), _ptr(roughness),
              ctypes.addressof(position_host), ctypes.addressof(rotation_host), fx, fy, far, near,
              ctypes.addressof(bg_host), initial_pair_capacity, *[t.data_ptr() for t in out]]
    return dict(zip(_FLASHGS_ORDER, values)), out, [position_host, rotation_host, bg_host]


def flashgs_forward(
    positions: torch.Tensor,
    shs: torch.Tensor,
    colors: torch.Tensor,
    opacities: torch.Tensor,
    covariance: torch.Tensor,
    scales: torch.Tensor,
    rotations: torch.Tensor,
    specular: torch.Tensor,
    roughness: torch.Tensor,
    *,
    width: int,
    height: int,
    use_sh: bool,
    camera_position: Sequence[float],
    camera_rotation: Sequence[float],
    focal_x: float,
    focal_y: float,
    z_far: float = 100.0,
    z_near: float = 0.01,
    background: Sequence[float] = (0.0, 0.0, 0.0),
    scale_modifier: float = 1.0,
    initial_pair_capacity: int = 1 << 20,
    context: NativeRendererContext,
    out: FlashgsOutputs | None = None,
    tile_rows: tuple[int, int] | None = None,
) -> FlashgsOutputs:
    """Deterministic FlashGS 16x16 forward; outputs are channel-first maps.

    tile_rows=(begin, end) renders only 16x16 tile rows [begin, end) (library
    extension for sharding one frame by strips): those rows are identical to a
    full-frame call, the other output rows are left untouched.
    """
    named, out, keep = _flashgs_arguments(
        positions, shs, colors, opacities, covariance, scales, rotations, specular, roughness, width=width,
        height=height, use_sh=use_sh, camera_position=camera_position, camera_rotation=camera_rotation,
        focal_x=focal_x, focal_y=focal_y, z_far=z_far, z_near=z_near, background=background,
        scale_modifier=scale_modifier, initial_pair_capacity=initial_pair_capacity, out=out)
    error = error_buffer()
    if tile_rows is not None:
        call = context.library.hs_b200_flashgs_forward_rows_f32_v1
        prefix = (context.handle, int(tile_rows[0]), int(tile_rows[1]))
    else:
        call = context.library.hs_flashgs_forward_f32_v1
        prefix = (context.handle,)
    status = call(*prefix, *[named[k] for k in _FLASHGS_ORDER], error, len(error))
    del keep
    check_status(status, "hs_b200_flashgs_forward_rows_f32_v1" if tile_rows is not None else
                 "hs_flashgs_forward_f32_v1", error)
    return out


def flashgs_forward_many(calls: Sequence[dict[str, Any]], *, stream: int | None = None) -> list[FlashgsOutputs]:
    """Independent FlashGS calls run concurrently (hs_b200_flashgs_forward_many_v2).

    Each item holds the arguments of one flashgs_forward call by name (the
    nine input tensors as ``positions`` ... ``roughness``, the keywords, and
    ``context``, distinct per item; ``tile_rows`` optional). ``stream`` is a
    raw cudaStream_t (default: the legacy default stream, like the v1 calls).
    Outputs are identical to calling flashgs_forward item by item.
    """
    structs, outs, keep = [], [], []
    library = None
    for item in calls:
        item = dict(item)
        context = item.pop("context")
        rows = item.pop("tile_rows", None)
        named, out, hold = _flashgs_arguments(**item)
        keep.append(hold)
        library = context.library
        structs.append(native_runtime.FlashgsCallV2(handle=context.handle, **named,
                                                    **_rows_fields(rows)))
        outs.append(out)
    if not structs:
        return []
    array = (native_runtime.FlashgsCallV2 * len(structs))(*structs)
    error = error_buffer()
    status = library.hs_b200_flashgs_forward_many_v2(array, len(structs), stream, error, len(error))
    del keep
    check_status(status, "hs_b200_flashgs_forward_many_v2", error)
    return outs


def _rows_fields(rows: tuple[int, int] | None) -> dict[str, int]:
    if rows is None:
        return {"tile_row_begin": 0, "tile_row_end": 0xFFFFFFFF}
    begin, end = int(rows[0]), int(rows[1])
    # an explicit strip end of UINT32_MAX is out of range, as in the rows entries
    return {"tile_row_begin": begin, "tile_row_end": 0xFFFFFFFE if end == 0xFFFFFFFF else end}


def _rasterizer_arguments(
    background: torch.Tensor,
    means3d: torch.Tensor,
    colors: torch.Tensor,
    opacities: torch.Tensor,
    scales: torch.Tensor,
    rotations: torch.Tensor,
    viewmatrix: torch.Tensor,
    projmatrix: torch.Tensor,
    camera_position: torch.Tensor,
    *,
    width: int,
    height: int,
    scale_modifier: float,
    tan_fovx: float,
    tan_fovy: float,
    prefiltered: bool = False,
    out: RasterizerOutputs | None = None,
) -> tuple[dict[str, Any], RasterizerOutputs]:
    """Checks one standard call; returns its named ABI arguments and outputs."""
    if isinstance(width, bool) or not isinstance(width, int) or width <= 0:
        raise ValueError("width must be a positive CPU integer")
    if isinstance(height, bool) or not isinstance(height, int) or height <= 0:
        raise ValueError("height must be a positive CPU integer")
    if not isinstance(prefiltered, bool):
        raise TypeError("prefiltered must be bool")
    count = int(means3d.shape[0])
    for name, value, shape in (
        ("background", background, (5,)),
        ("means3d", means3d, (count, 3)),
        ("colors", colors, (count, 5)),
        ("opacities", opacities, (count, 1)),
        ("scales", scales, (count, 2)),
        ("rotations", rotations, (count, 4)),
        ("viewmatrix", viewmatrix, (4, 4)),
        ("projmatrix", projmatrix, (4, 4)),
        ("camera_position", camera_position, (3,)),
    ):
        _check_tensor(name, value, shape)
    scale = _finite("scale_modifier", scale_modifier, positive=True)
    fovx = _finite("tan_fovx", tan_fovx, positive=True)
    fovy = _finite("tan_fovy", tan_fovy, positive=True)
    device = means3d.device
    if out is None:
        f = dict(dtype=torch.float32, device=device)
        out = RasterizerOutputs(
            torch.empty((5, height, width), **f),
            torch.empty((7, height, width), **f),
            torch.empty((count, 1), **f),
            torch.empty((count,), dtype=torch.int32, device=device),
            torch.empty((1,), dtype=torch.int32, device=device),
        )
    values = [count, _ptr(background), width, height, _ptr(means3d), _ptr(colors), _ptr(opacities),
              _ptr(scales), scale, _ptr(rotations), _ptr(viewmatrix), _ptr(projmatrix), _ptr(camera_position),
              fovx, fovy, int(prefiltered), *[t.data_ptr() for t in out]]
    return dict(zip(_RASTERIZER_ORDER, values)), out


def rasterize_forward(
    background: torch.Tensor,
    means3d: torch.Tensor,
    colors: torch.Tensor,
    opacities: torch.Tensor,
    scales: torch.Tensor,
    rotations: torch.Tensor,
    viewmatrix: torch.Tensor,
    projmatrix: torch.Tensor,
    camera_position: torch.Tensor,
    *,
    width: int,
    height: int,
    scale_modifier: float,
    tan_fovx: float,
    tan_fovy: float,
    prefiltered: bool = False,
    context: NativeRendererContext,
    out: RasterizerOutputs | None = None,
    tile_rows: tuple[int, int] | None = None,
) -> RasterizerOutputs:
    """Standard five-channel 2DGS forward (color[5,H,W], aux[7,H,W], ...).

    tile_rows=(begin, end): render only those 16x16 tile rows, as in
    flashgs_forward (library extension).
    """
    named, out = _rasterizer_arguments(
        background, means3d, colors, opacities, scales, rotations, viewmatrix, projmatrix, camera_position,
        width=width, height=height, scale_modifier=scale_modifier, tan_fovx=tan_fovx, tan_fovy=tan_fovy,
        prefiltered=prefiltered, out=out)
    error = error_buffer()
    if tile_rows is not None:
        call = context.library.hs_b200_rasterizer_forward_rows_f32_v1
        prefix = (context.handle, int(tile_rows[0]), int(tile_rows[1]))
    else:
        call = context.library.hs_rasterizer_forward_f32_v1
        prefix = (context.handle,)
    status = call(*prefix, *[named[k] for k in _RASTERIZER_ORDER], error, len(error))
    check_status(status, "hs_b200_rasterizer_forward_rows_f32_v1" if tile_rows is not None else
                 "hs_rasterizer_forward_f32_v1", error)
    return out


def rasterize_forward_many(calls: Sequence[dict[str, Any]], *,
                           stream: int | None = None) -> list[RasterizerOutputs]:
    """Independent standard calls run concurrently (hs_b200_rasterizer_forward_many_v2).

    Each item holds the arguments of one rasterize_forward call by name (the
    nine tensors ``background`` ... ``camera_position``, the keywords and a
    distinct ``context``; ``tile_rows`` optional). ``stream`` as in
    flashgs_forward_many. Outputs are identical to calling rasterize_forward
    item by item.
    """
    structs, outs = [], []
    library = None
    for item in calls:
        item = dict(item)
        context = item.pop("context")
        rows = item.pop("tile_rows", None)
        named, out = _rasterizer_arguments(**item)
        library = context.library
        structs.append(native_runtime.RasterizerCallV2(handle=context.handle, **named, **_rows_fields(rows)))
        outs.append(out)
    if not structs:
        return []
    array = (native_runtime.RasterizerCallV2 * len(structs))(*structs)
    error = error_buffer()
    status = library.hs_b200_rasterizer_forward_many_v2(array, len(structs), stream, error, len(error))
    check_status(status, "hs_b200_rasterizer_forward_many_v2", error)
    return outs


def rasterize_forward_noalloc(
    background: torch.Tensor,
    means3d: torch.Tensor,
    colors: torch.Tensor,
    opacities: torch.Tensor,
    scales: torch.Tensor,
    rotations: torch.Tensor,
    viewmatrix: torch.Tensor,
    projmatrix: torch.Tensor,
    camera_position: torch.Tensor,
    *,
    width: int,
    height: int,
    scale_modifier: float,
    tan_fovx: float,
    tan_fovy: float,
    prefiltered: bool = False,
    out: RasterizerOutputs | None = None,
    library: ctypes.CDLL | None = None,
) -> RasterizerOutputs:
    """rasterize_forward through hs_b200_rasterizer_forward_noalloc_f32_v1:
    no context, no allocation inside the library (small views only: at most
    16384 Gaussians, 4096 tiles and 262144 emitted pairs). The entry point
    runs on the legacy default stream, so work queued on a non-default torch
    stream (which may have produced the inputs) is waited for first."""
    library = library if library is not None else load_native_library()
    named, out = _rasterizer_arguments(
        background, means3d, colors, opacities, scales, rotations, viewmatrix, projmatrix, camera_position,
        width=width, height=height, scale_modifier=scale_modifier, tan_fovx=tan_fovx, tan_fovy=tan_fovy,
        prefiltered=prefiltered, out=out)
    stream = torch.cuda.current_stream(means3d.device)
    if stream.cuda_stream != 0:
        stream.synchronize()
    error = error_buffer()
    status = library.hs_b200_rasterizer_forward_noalloc_f32_v1(
        means3d.device.index if means3d.device.index is not None else torch.cuda.current_device(),
        *[named[k] for k in _RASTERIZER_ORDER], error, len(error))
    check_status(status, "hs_b200_rasterizer_forward_noalloc_f32_v1", error)
    return out


def flashgs_prepare_host(
    opacity_raw, scaling_raw, rotation_raw, specular_raw, roughness_raw, *, library: ctypes.CDLL | None = None
) -> dict[str, Any]:
    """Host FlashGS activation of raw NPZ arrays (numpy float32 in and out)."""
    import numpy as np

    lib = library if library is not None else load_native_library()
    arrays = [np.ascontiguousarray(a, dtype=np.float32) for a in
              (opacity_raw, scaling_raw, rotation_raw, specular_raw, roughness_raw)]
    count = int(arrays[0].shape[0])
    shapes = [(count, 1), (count, 2), (count, 4), (count, 1), (count, 1)]
    for a, shape in zip(arrays, shapes):
        if a.shape != shape:
            raise ValueError(f"expected shape {shape}, got {a.shape}")
    out = {
        "opacity": np.empty((count, 1), np.float32),
        "scaling": np.empty((count, 2), np.float32),
        "rotation": np.empty((count, 4), np.float32),
        "covariance": np.empty((count, 6), np.float32),
        "specular": np.empty((count, 1), np.float32),
        "roughness": np.empty((count, 1), np.float32),
    }
    error = error_buffer()
    status = lib.hs_flashgs_prepare_npz_host_f32_v1(
        count, *[a.ctypes.data for a in arrays], *[v.ctypes.data for v in out.values()], error, len(error)
    )
    check_status(status, "hs_flashgs_prepare_npz_host_f32_v1", error)
    return out


def _elementwise(symbol: str, library: ctypes.CDLL | None, *args: Any) -> None:
    lib = library if library is not None else load_native_library()
    error = error_buffer()
    status = getattr(lib, symbol)(*args, error, len(error))
    check_status(status, symbol, error)


def precise_exp(x: torch.Tensor, *, library: ctypes.CDLL | None = None) -> torch.Tensor:
    out = torch.empty_like(x)
    _elementwise("hs_rasterizer_precise_exp_f32_v1", library, _ptr(x), _ptr(out), x.numel())
    return out


def precise_sigmoid(x: torch.Tensor, *, library: ctypes.CDLL | None = None) -> torch.Tensor:
    out = torch.empty_like(x)
    _elementwise("hs_rasterizer_precise_sigmoid_f32_v1", library, _ptr(x), _ptr(out), x.numel())
    return out


def precise_normalize4(x: torch.Tensor, *, library: ctypes.CDLL | None = None) -> torch.Tensor:
    _check_tensor("input", x, (int(x.shape[0]), 4))
    out = torch.empty_like(x)
    _elementwise("hs_rasterizer_precise_normalize4_f32_v1", library, _ptr(x), _ptr(out), x.shape[0])
    return out


def precise_fuse_maps(base_rgb: torch.Tensor, reflection_rgb: torch.Tensor, specular: torch.Tensor, *,
                      library: ctypes.CDLL | None = None) -> dict[str, torch.Tensor]:
    """dif = base*(1-s), ref = (refl*s)*2, rgb = dif + 0.5*ref (math.py:301-311)."""
    pixels = base_rgb.numel() // 3
    diffuse = torch.empty_like(base_rgb)
    final = torch.empty_like(base_rgb)
    stored = torch.empty_like(base_rgb)
    _elementwise("hs_rasterizer_precise_fuse_maps_f32_v1", library, _ptr(base_rgb), _ptr(reflection_rgb),
                 _ptr(specular), _ptr(diffuse), _ptr(final), _ptr(stored), pixels)
    return {"rgb_map": final, "dif_rgb_map": diffuse, "ref_rgb_map": stored}


def precise_fuse_maps_planar(base_rgb: torch.Tensor, reflection_rgb: torch.Tensor, specular: torch.Tensor, *,
                             library: ctypes.CDLL | None = None) -> dict[str, torch.Tensor]:
    """precise_fuse_maps of channel-first inputs: base_rgb and reflection_rgb
    [3,H,W] (views of a raster call's colour planes), specular [1,H,W] or
    [H,W]; returns the same [H,W,3] maps as precise_fuse_maps of their
    HWC transposes (hs_b200_precise_fuse_maps_planar_f32_v1)."""
    if base_rgb.shape[0] != 3 or reflection_rgb.shape != base_rgb.shape:
        raise ValueError("base_rgb and reflection_rgb must be [3,H,W]")
    for name, t in (("base_rgb", base_rgb), ("reflection_rgb", reflection_rgb), ("specular", specular)):
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
    h, w = int(base_rgb.shape[1]), int(base_rgb.shape[2])
    if specular.numel() != h * w:
        raise ValueError("specular must hold one value per pixel")
    f = dict(dtype=torch.float32, device=base_rgb.device)
    diffuse, final, stored = (torch.empty((h, w, 3), **f) for _ in range(3))
    _elementwise("hs_b200_precise_fuse_maps_planar_f32_v1", library, _ptr(base_rgb), _ptr(reflection_rgb),
                 _ptr(specular), _ptr(diffuse), _ptr(final), _ptr(stored), h * w)
    return {"rgb_map": final, "dif_rgb_map": diffuse, "ref_rgb_map": stored}


def precise_sh_colors5(sh: torch.Tensor, points: torch.Tensor, center: torch.Tensor, specular: torch.Tensor,
                       roughness: torch.Tensor, degree: int, *, library: ctypes.CDLL | None = None) -> torch.Tensor:
    """[P,5] = [precise_sh_to_rgb(sh, precise_direction(points, center), degree),
    specular, roughness] in one pass (hs_b200_precise_sh_colors5_f32_v1)."""
    sh = sh.contiguous()
    count = int(points.shape[0])
    out = torch.empty((count, 5), dtype=torch.float32, device=points.device)
    _elementwise("hs_b200_precise_sh_colors5_f32_v1", library, _ptr(sh), int(sh.shape[-1]), int(degree),
                 _ptr(points), _ptr(center), _ptr(specular), _ptr(roughness), count, _ptr(out))
    return out


def precise_sh_to_rgb(sh: torch.Tensor, directions: torch.Tensor, degree: int, *,
                      library: ctypes.CDLL | None = None) -> torch.Tensor:
    """sh is [P,3,C] (channel-major), directions [P,3]; returns [P,3]."""
    sh = sh.contiguous()
    count = int(directions.shape[0])
    out = torch.empty((count, 3), dtype=torch.float32, device=directions.device)
    _elementwise("hs_rasterizer_precise_sh_to_rgb_f32_v1", library, _ptr(sh), _ptr(directions), count,
                 int(sh.shape[-1]), int(degree), _ptr(out))
    return out


def precise_direction(points: torch.Tensor, center: torch.Tensor, *,
                      library: ctypes.CDLL | None = None) -> torch.Tensor:
    out = torch.empty_like(points)
    _elementwise("hs_rasterizer_precise_direction_f32_v1", library, _ptr(points), _ptr(center),
                 points.shape[0], _ptr(out))
    return out


def precise_reflection_prefix(rotation_wxyz: torch.Tensor, *, library: ctypes.CDLL | None = None) -> torch.Tensor:
    count = int(rotation_wxyz.shape[0])
    out = torch.empty((count, 3, 3), dtype=torch.float32, device=rotation_wxyz.device)
    _elementwise("hs_rasterizer_precise_reflection_prefix_f32_v1", library, _ptr(rotation_wxyz), count, _ptr(out))
    return out


def precise_reflection_suffix(xyz: torch.Tensor, camera_center: torch.Tensor, normal_raw: torch.Tensor, *,
                              library: ctypes.CDLL | None = None) -> torch.Tensor:
    count = int(xyz.shape[0])
    out = torch.empty((count, 36), dtype=torch.float32, device=xyz.device)
    _elementwise("hs_rasterizer_precise_reflection_suffix_f32_v1", library, _ptr(xyz), _ptr(camera_center),
                 _ptr(normal_raw), count, _ptr(out))
    return out


def precise_disk_rotation(rotation_wxyz: torch.Tensor, *, library: ctypes.CDLL | None = None) -> torch.Tensor:
    count = int(rotation_wxyz.shape[0])
    out = torch.empty((count, 3, 3), dtype=torch.float32, device=rotation_wxyz.device)
    _elementwise("hs_rasterizer_precise_disk_rotation_f32_v1", library, _ptr(rotation_wxyz), count, _ptr(out))
    return out


# ---------------------------------------------------------------- reflection trace


def gaussian_disks(xyz: torch.Tensor, rotation_raw: torch.Tensor, scaling: torch.Tensor, *,
                   library: ctypes.CDLL | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """The trace scene of a Gaussian group (math.py:253-298): each Gaussian's
    disk as the square of +-3 sigma in its plane, two triangles
    (4g, 4g+1, 4g+2) and (4g+1, 4g+2, 4g+3) over the corners (-3, 3),
    (-3, -3), (3, 3), (3, -3). The rotation is hs_rasterizer_precise_disk_rotation_f32_v1
    of the raw quaternions; corner = (R[:, 0] s0) sx + (R[:, 1] s1) sy + xyz
    in float32 (the reference forms the same products with a framework
    matmul). Returns vertices [4P, 3] float32 and triangles [2P, 3] int32."""
    count = int(xyz.shape[0])
    _check_tensor("xyz", xyz, (count, 3))
    _check_tensor("rotation_raw", rotation_raw, (count, 4))
    _check_tensor("scaling", scaling, (count, 2))
    rot = precise_disk_rotation(rotation_raw, library=library)
    col0 = rot[:, :, 0] * scaling[:, 0:1]
    col1 = rot[:, :, 1] * scaling[:, 1:2]
    corners = torch.tensor([[-3.0, 3.0], [-3.0, -3.0], [3.0, 3.0], [3.0, -3.0]], dtype=torch.float32,
                           device=xyz.device)
    vertices = (col0[:, None, :] * corners[None, :, 0:1] + col1[:, None, :] * corners[None, :, 1:2]) + \
        xyz[:, None, :]
    idx = torch.arange(count * 4, dtype=torch.int32, device=xyz.device).view(count, 4)
    triangles = torch.stack((idx[:, :3], idx[:, 1:]), dim=1).reshape(-1, 3).contiguous()
    return vertices.reshape(-1, 3).contiguous(), triangles


def build_trace_scene(vertices: torch.Tensor, triangles: torch.Tensor, *, scene_signature: int = 1,
                      rebuild: bool = True, context: NativeRendererContext) -> int:
    """hs_optix_build_scene_v1 (reference ops/optix.py build_optix_scene):
    the trace scene of vertices [V, 3] float32 and triangles [T, 3] int32;
    returns the device status word (0)."""
    vertex_count, triangle_count = int(vertices.shape[0]), int(triangles.shape[0])
    _check_tensor("vertices", vertices, (vertex_count, 3))
    _check_tensor("triangles", triangles, (triangle_count, 3), dtype=torch.int32)
    status = torch.full((1,), -1, dtype=torch.int32, device=vertices.device)
    error = error_buffer()
    rc = context.library.hs_optix_build_scene_v1(context.handle, _ptr(vertices), vertex_count, _ptr(triangles),
                                                 triangle_count, int(scene_signature), int(bool(rebuild)),
                                                 _ptr(status), error, len(error))
    check_status(rc, "hs_optix_build_scene_v1", error)
    return int(status.item())


def trace_reflection(ray_origins: torch.Tensor, ray_directions: torch.Tensor, background: torch.Tensor,
                     means3d: torch.Tensor, shs: torch.Tensor, others: torch.Tensor, opacities: torch.Tensor,
                     scales: torch.Tensor, rotations: torch.Tensor, viewmatrix: torch.Tensor,
                     projmatrix: torch.Tensor, camera_position: torch.Tensor, *, degree: int,
                     scale_modifier: float = 1.0, start_from_first: bool = False, max_trace_depth: int = 0,
                     specular_threshold: float = 0.0, use_others: bool = True,
                     context: NativeRendererContext, out: TraceOutputs | None = None) -> TraceOutputs:
    """hs_optix_trace_f32_v1 (reference ops/optix.py trace_optix): one ray per
    Gaussian of the traced group against the scene built by
    build_trace_scene; shs is [P, M, 3]."""
    count = int(ray_origins.shape[0])
    coefficients = int(shs.shape[1])
    for name, value, shape in (("ray_origins", ray_origins, (count, 3)), ("ray_directions", ray_directions, (count, 3)),
                               ("background", background, (3,)), ("means3d", means3d, (count, 3)),
                               ("shs", shs, (count, coefficients, 3)), ("others", others, (count, 2)),
                               ("opacities", opacities, (count, 1)), ("scales", scales, (count, 2)),
                               ("rotations", rotations, (count, 4)), ("viewmatrix", viewmatrix, (4, 4)),
                               ("projmatrix", projmatrix, (4, 4)), ("camera_position", camera_position, (3,))):
        _check_tensor(name, value, shape)
    if isinstance(degree, bool) or not isinstance(degree, int) or degree not in range(4):
        raise ValueError("degree must be an integer in [0, 3]")
    if max_trace_depth not in (0, 1) or isinstance(max_trace_depth, bool):
        raise ValueError("max_trace_depth must be 0 or 1")
    if out is None:
        f = dict(dtype=torch.float32, device=ray_origins.device)
        out = TraceOutputs(torch.empty((count, 3), **f), torch.empty((count, 1), **f), torch.empty((count, 1), **f),
                           torch.empty((count, 3), **f), torch.empty((count, 1), **f), torch.empty((count, 2), **f),
                           torch.empty((count, 32), **f), torch.empty((count, 1), **f))
    error = error_buffer()
    rc = context.library.hs_optix_trace_f32_v1(
        context.handle, count, _ptr(ray_origins), _ptr(ray_directions), _ptr(background), _ptr(means3d), _ptr(shs),
        coefficients, degree, _ptr(others), _ptr(opacities), _ptr(scales), _finite("scale_modifier", scale_modifier),
        _ptr(rotations), _ptr(viewmatrix), _ptr(projmatrix), _ptr(camera_position), int(bool(start_from_first)),
        int(max_trace_depth), _finite("specular_threshold", specular_threshold), int(bool(use_others)),
        *[_ptr(t) for t in out], error, len(error))
    check_status(rc, "hs_optix_trace_f32_v1", error)
    return out


# ---------------------------------------------------------------- postprocess


def precise_general_inverse(matrix: torch.Tensor, *, context: NativeRendererContext) -> torch.Tensor:
    """Inverse of a row-major 3x3 or 4x4 device matrix by the reference's LU
    route (hs_rasterizer_precise_general_inverse_f32_v2)."""
    n = int(matrix.shape[0])
    _check_tensor("matrix", matrix, (n, n))
    matrix = matrix.contiguous()
    out = torch.empty_like(matrix)
    error = error_buffer()
    status = context.library.hs_rasterizer_precise_general_inverse_f32_v2(context.handle, _ptr(matrix), n,
                                                                          _ptr(out), error, len(error))
    check_status(status, "hs_rasterizer_precise_general_inverse_f32_v2", error)
    return out


def precise_matmul_nt_n3k3(left: torch.Tensor, right: torch.Tensor, *,
                           context: NativeRendererContext) -> torch.Tensor:
    """left[N,3] @ right[3,3]^T rounded as the reference's TF32 tensor-op
    cuBLAS GEMM rounds it (hs_rasterizer_precise_matmul_nt_n3k3_f32_v2; an
    MMA kernel in this library)."""
    count = int(left.shape[0])
    _check_tensor("left", left, (count, 3))
    _check_tensor("right", right, (3, 3))
    left, right = left.contiguous(), right.contiguous()
    out = torch.empty_like(left)
    error = error_buffer()
    status = context.library.hs_rasterizer_precise_matmul_nt_n3k3_f32_v2(context.handle, _ptr(left), _ptr(right),
                                                                        count, _ptr(out), error, len(error))
    check_status(status, "hs_rasterizer_precise_matmul_nt_n3k3_f32_v2", error)
    return out


def session_focal_from_fov(length: int, fov: float) -> np.float32:
    """The session's FP32 focal length from a field of view (math.py:339-348)."""
    fov32 = np.float32(fov)
    half = np.divide(fov32, np.float32(2.0), dtype=np.float32)
    denominator = np.float32(2.0 * math.tan(float(half)))
    return np.divide(np.float32(length), denominator, dtype=np.float32)


def postprocess_camera(width: int, height: int, fov_x: float, fov_y: float, world_view_transform: torch.Tensor, *,
                       context: NativeRendererContext) -> dict[str, torch.Tensor]:
    """The per-view matrices of the standard postprocess (math.py:354-401,
    426-433) on the device: the inverse intrinsics, the camera-to-world
    rotation and origin, and the normal rotation world_view_transform[:3,:3]^T.
    world_view_transform is the [4,4] matrix as the session stores it."""
    _check_tensor("world_view_transform", world_view_transform, (4, 4))
    f = np.float32
    intrinsics = np.array([[session_focal_from_fov(width, fov_x), f(0.0), np.divide(f(width), f(2.0), dtype=f)],
                           [f(0.0), session_focal_from_fov(height, fov_y), np.divide(f(height), f(2.0), dtype=f)],
                           [f(0.0), f(0.0), f(1.0)]], dtype=f)
    device = world_view_transform.device
    inverse_intrinsics = precise_general_inverse(torch.from_numpy(intrinsics).to(device), context=context)
    c2w = precise_general_inverse(world_view_transform.transpose(0, 1).contiguous(), context=context)
    return {"inverse_intrinsics": inverse_intrinsics, "rotation": c2w[:3, :3].contiguous(),
            "origin": c2w[:3, 3].contiguous(),
            "normal_rotation": world_view_transform[:3, :3].transpose(0, 1).contiguous()}


def pixel_rays(width: int, height: int, inverse_intrinsics: torch.Tensor, rotation: torch.Tensor, *,
               context: NativeRendererContext, out: torch.Tensor | None = None,
               scratch: torch.Tensor | None = None) -> torch.Tensor:
    """World-space rays [H*W,3] of every pixel, ((x, y, 1) @ K^-T) @ R^T with
    the reference's TF32 GEMM rounding for each product, in one tensor-core
    kernel (hs_b200_pixel_rays_f32_v1; `scratch` is accepted for the ABI and
    not written)."""
    _check_tensor("inverse_intrinsics", inverse_intrinsics, (3, 3))
    _check_tensor("rotation", rotation, (3, 3))
    f = dict(dtype=torch.float32, device=rotation.device)
    rays = out if out is not None else torch.empty((height * width, 3), **f)
    work = scratch if scratch is not None else torch.empty((height * width, 3), **f)
    for name, t in (("out", rays), ("scratch", work)):
        _check_tensor(name, t, (height * width, 3))
    error = error_buffer()
    status = context.library.hs_b200_pixel_rays_f32_v1(context.handle, int(width), int(height),
                                                        _ptr(inverse_intrinsics.contiguous()),
                                                        _ptr(rotation.contiguous()), _ptr(work), _ptr(rays),
                                                        error, len(error))
    check_status(status, "hs_b200_pixel_rays_f32_v1", error)
    return rays


def postprocess_camera_rays(width: int, height: int, fov_x: float, fov_y: float, world_view_transform: torch.Tensor,
                            *, context: NativeRendererContext, stream: int | None = None,
                            camera: torch.Tensor | None = None, rays: torch.Tensor | None = None
                            ) -> dict[str, torch.Tensor]:
    """postprocess_camera and pixel_rays in one call on `stream` (a raw
    cudaStream_t; None = the legacy default stream), so that a session can
    run them beside the raster calls (hs_b200_postprocess_camera_f32_v1).
    Returns the same matrices as postprocess_camera (views of one 30-float
    buffer) and the rays."""
    _check_tensor("world_view_transform", world_view_transform, (4, 4))
    device = world_view_transform.device
    f = dict(dtype=torch.float32, device=device)
    camera = camera if camera is not None else torch.empty(30, **f)
    rays = rays if rays is not None else torch.empty((height * width, 3), **f)
    _check_tensor("camera", camera, (30,))
    _check_tensor("rays", rays, (height * width, 3))
    error = error_buffer()
    status = context.library.hs_b200_postprocess_camera_f32_v1(
        context.handle, int(width), int(height), float(fov_x), float(fov_y), _ptr(world_view_transform.contiguous()),
        _ptr(camera), _ptr(rays), stream, error, len(error))
    check_status(status, "hs_b200_postprocess_camera_f32_v1", error)
    return {"inverse_intrinsics": camera[0:9].view(3, 3), "rotation": camera[9:18].view(3, 3),
            "origin": camera[18:21], "normal_rotation": camera[21:30].view(3, 3), "rays": rays}


STANDARD_MAPS = ("rgb_map", "acc_map", "dpt_map", "norm_map", "surf_norm_map", "dist_map", "spec_map", "rough_map")
STANDARD_MAP_CHANNELS = (3, 1, 1, 3, 3, 1, 1, 1)


def standard_postprocess(color: torch.Tensor, auxiliary: torch.Tensor, rays: torch.Tensor, origin: torch.Tensor,
                         normal_rotation: torch.Tensor, *, depth_ratio: float = 0.0,
                         library: ctypes.CDLL | None = None) -> dict[str, torch.Tensor]:
    """postprocess_raster (math.py:426-463) of a standard raster call's
    color[5,H,W] and auxiliary[7,H,W] in one pass
    (hs_b200_standard_postprocess_f32_v1). Returns the session's maps, each
    [1,H*W,C]."""
    h, w = int(color.shape[1]), int(color.shape[2])
    _check_tensor("color", color, (5, h, w))
    _check_tensor("auxiliary", auxiliary, (7, h, w))
    _check_tensor("rays", rays, (h * w, 3))
    _check_tensor("origin", origin, (3,))
    _check_tensor("normal_rotation", normal_rotation, (3, 3))
    ratio = _finite("depth_ratio", depth_ratio)
    f = dict(dtype=torch.float32, device=color.device)
    maps = {name: torch.empty((1, h * w, c), **f) for name, c in zip(STANDARD_MAPS, STANDARD_MAP_CHANNELS)}
    _elementwise("hs_b200_standard_postprocess_f32_v1", library, w, h, _ptr(color.contiguous()),
                 _ptr(auxiliary.contiguous()), _ptr(rays.contiguous()), _ptr(origin.contiguous()),
                 _ptr(normal_rotation.contiguous()), ratio, *[_ptr(maps[n]) for n in STANDARD_MAPS])
    return maps


def flashgs_postprocess(raster: FlashgsOutputs, normal_rotation: torch.Tensor, *,
                        library: ctypes.CDLL | None = None) -> dict[str, torch.Tensor]:
    """_flashgs_postprocess (renderer.py:176-202) of a FlashGS forward in one
    pass (hs_b200_flashgs_postprocess_f32_v1); maps are [1,H*W,C]."""
    h, w = int(raster.alpha.shape[1]), int(raster.alpha.shape[2])
    _check_tensor("normal_rotation", normal_rotation, (3, 3))
    f = dict(dtype=torch.float32, device=raster.alpha.device)
    names = ("rgb_map", "acc_map", "dpt_map", "norm_map", "surf_norm_map", "dist_map", "spec_map")
    channels = (3, 1, 1, 3, 3, 1, 1)
    maps = {n: torch.empty((1, h * w, c), **f) for n, c in zip(names, channels)}
    _elementwise("hs_b200_flashgs_postprocess_f32_v1", library, w, h, _ptr(raster.color.contiguous()),
                 _ptr(raster.other.contiguous()), _ptr(raster.depth.contiguous()), _ptr(raster.alpha.contiguous()),
                 _ptr(raster.normal.contiguous()), _ptr(normal_rotation.contiguous()),
                 *[_ptr(maps[n]) for n in names])
    return maps


# ---------------------------------------------------------------- one view


class StandardViewOutputs(NamedTuple):
    """Everything standard_view writes: both raster calls' outputs, the
    colours they took, the reflection preparation, the trace and its ray
    origins and directions (when traced, else None), the fused maps and, with
    the postprocess, its camera terms and maps (else None)."""
    base: RasterizerOutputs
    reflection: RasterizerOutputs
    base_colors: torch.Tensor
    reflection_colors: torch.Tensor
    reflection_rotation: torch.Tensor
    reflection_normal: torch.Tensor
    reflection_rays: torch.Tensor
    ray_origins: torch.Tensor
    ray_directions: torch.Tensor
    trace: TraceOutputs | None
    fused: dict[str, torch.Tensor]
    camera: dict[str, torch.Tensor] | None
    maps: dict[str, torch.Tensor] | None


def _event_handle(event: torch.cuda.Event | None) -> int | None:
    """The cudaEvent_t of a torch event (created by a first record if torch
    has not created it yet)."""
    if event is None:
        return None
    if not event.cuda_event:
        event.record()
    return int(event.cuda_event)


def standard_view(base: dict[str, torch.Tensor], reflection: dict[str, torch.Tensor], viewmatrix: torch.Tensor,
                  projmatrix: torch.Tensor, camera_position: torch.Tensor, background: torch.Tensor, *,
                  width: int, height: int, tan_fovx: float, tan_fovy: float, sh_degree: int,
                  base_context: NativeRendererContext, reflection_context: NativeRendererContext,
                  trace: dict[str, Any] | None = None, postprocess: dict[str, float] | None = None,
                  stream: int | None = None, raster_begin_event: torch.cuda.Event | None = None,
                  out: StandardViewOutputs | None = None) -> StandardViewOutputs:
    """One view of the standard session (render_hybridsplat_view,
    renderer.py:232-341, and postprocess_raster, math.py:426-463) in one call
    (hs_b200_standard_view_v2).

    ``base`` holds the activated base group (``means3d``, ``opacities``,
    ``scales``, ``rotations``, ``specular``, ``roughness``) and its SH ``sh``
    [P,3,C] (channel-major); ``reflection`` the activated reflection group,
    its raw quaternions ``rotations_raw`` and, unless traced, its colours
    ``rgb`` [R,3]. ``trace`` (optional) traces the reflection colours on
    reflection_context's built scene: ``background`` [3], ``shs`` [R,C,3],
    ``others`` [R,2], ``degree``, and optionally ``use_others`` (True),
    ``max_trace_depth`` (0), ``specular_threshold`` (0.0), as trace_reflection.
    ``postprocess`` (optional) adds the raw-map postprocess: ``fov_x``,
    ``fov_y`` and ``depth_ratio`` (0.0). ``background`` is the raster calls'
    [5]. ``stream`` as in rasterize_forward_many. ``raster_begin_event``
    (optional) is recorded when both calls' binning is done, before the tile
    renderers. ``out`` (optional) is the result of an earlier call with the
    same sizes, trace and postprocess choice, whose tensors receive the
    outputs: an untraced view whose arguments and buffers repeat those of one
    of the context's last calls replays as one captured graph on a
    non-default ``stream`` (hs_b200_view_graph_stats_v1), so reusing a few
    output sets lets a sequence of views replay. Every output equals that of
    the same steps called one by one.
    """
    if base_context is reflection_context:
        raise ValueError("standard_view needs two distinct contexts")
    device = viewmatrix.device
    f = dict(dtype=torch.float32, device=device)

    def take(name, existing, shape):
        if out is None:
            return torch.empty(shape, **f)
        if existing is None:
            raise ValueError(f"out has no {name}")
        _check_tensor(f"out {name}", existing, shape)
        return existing

    sh = base["sh"].contiguous()
    nb, nr = int(base["means3d"].shape[0]), int(reflection["means3d"].shape[0])
    _check_tensor("base sh", sh, (nb, 3, int(sh.shape[-1])))
    _check_tensor("reflection rotations_raw", reflection["rotations_raw"], (nr, 4))
    if isinstance(sh_degree, bool) or not isinstance(sh_degree, int) or sh_degree not in range(4):
        raise ValueError("sh_degree must be an integer in [0, 3]")
    base_colors = take("base_colors", out and out.base_colors, (nb, 5))
    refl_colors = take("reflection_colors", out and out.reflection_colors, (nr, 5))
    for name, group, n in (("base", base, nb), ("reflection", reflection, nr)):
        _check_tensor(f"{name} specular", group["specular"], (n, 1))
        _check_tensor(f"{name} roughness", group["roughness"], (n, 1))
    common = dict(width=width, height=height, scale_modifier=1.0, tan_fovx=tan_fovx, tan_fovy=tan_fovy)
    named_b, out_b = _rasterizer_arguments(background, base["means3d"], base_colors, base["opacities"],
                                           base["scales"], base["rotations"], viewmatrix, projmatrix,
                                           camera_position, out=out and out.base, **common)
    named_r, out_r = _rasterizer_arguments(background, reflection["means3d"], refl_colors, reflection["opacities"],
                                           reflection["scales"], reflection["rotations"], viewmatrix, projmatrix,
                                           camera_position, out=out and out.reflection, **common)

    def group(named, g):
        return native_runtime.StandardGroupV2(
            count=named["point_count"], means3d=named["means3d"], opacities=named["opacities"],
            scales2=named["scales2"], rotations4=named["rotations4"], specular=_ptr(g["specular"]),
            roughness=_ptr(g["roughness"]), background5=named["background5"], colors5=named["colors5"],
            output_color5=named["output_color5"], output_aux7=named["output_aux7"],
            output_weight=named["output_weight"], output_radii=named["output_radii"],
            output_rendered=named["output_rendered"])

    rotation = take("reflection_rotation", out and out.reflection_rotation, (nr, 3, 3))
    normal = take("reflection_normal", out and out.reflection_normal, (nr, 3))
    rays = take("reflection_rays", out and out.reflection_rays, (nr, 36))
    origins = directions = None
    pixels = width * height
    fused = {k: take(k, out and out.fused.get(k), (height, width, 3)) for k in ("rgb_map", "dif_rgb_map", "ref_rgb_map")}
    view = native_runtime.StandardViewV2(
        struct_size=ctypes.sizeof(native_runtime.StandardViewV2), base_handle=base_context.handle,
        reflection_handle=reflection_context.handle, width=width, height=height, tan_fovx=named_b["tan_fovx"],
        tan_fovy=named_b["tan_fovy"], viewmatrix4x4=_ptr(viewmatrix), projmatrix4x4=_ptr(projmatrix),
        camera_position3=_ptr(camera_position), base=group(named_b, base), reflection=group(named_r, reflection),
        base_sh=_ptr(sh), sh_coefficients=int(sh.shape[-1]), sh_degree=sh_degree,
        reflection_rotation_raw4=_ptr(reflection["rotations_raw"]), reflection_rotation9=_ptr(rotation),
        reflection_normal3=_ptr(normal), reflection_rays36=_ptr(rays), fused_rgb3=_ptr(fused["rgb_map"]),
        diffuse_rgb3=_ptr(fused["dif_rgb_map"]), reflection_rgb_map3=_ptr(fused["ref_rgb_map"]), stream=stream)
    traced = None
    if trace is None:
        rgb = reflection["rgb"]
        _check_tensor("reflection rgb", rgb, (nr, 3))
        view.reflection_rgb3 = _ptr(rgb)
    else:
        shs = trace["shs"]
        coefficients = int(shs.shape[1])
        _check_tensor("trace background", trace["background"], (3,))
        _check_tensor("trace shs", shs, (nr, coefficients, 3))
        _check_tensor("trace others", trace["others"], (nr, 2))
        degree = trace["degree"]
        if isinstance(degree, bool) or not isinstance(degree, int) or degree not in range(4):
            raise ValueError("degree must be an integer in [0, 3]")
        depth = trace.get("max_trace_depth", 0)
        if depth not in (0, 1) or isinstance(depth, bool):
            raise ValueError("max_trace_depth must be 0 or 1")
        widths = (3, 1, 1, 3, 1, 2, 32, 1)
        traced = TraceOutputs(*(take(f"trace.{k}", out and out.trace and getattr(out.trace, k), (nr, c))
                                for k, c in zip(TraceOutputs._fields, widths)))
        origins = take("ray_origins", out and out.ray_origins, (nr, 3))
        directions = take("ray_directions", out and out.ray_directions, (nr, 3))
        view.trace = 1
        view.reflection_ray_origins3 = _ptr(origins)
        view.reflection_ray_directions3 = _ptr(directions)
        view.trace_background3 = _ptr(trace["background"])
        view.reflection_shs = _ptr(shs)
        view.trace_coefficients = coefficients
        view.trace_degree = degree
        view.reflection_others2 = _ptr(trace["others"])
        view.use_others = int(bool(trace.get("use_others", True)))
        view.max_trace_depth = int(depth)
        view.specular_threshold = _finite("specular_threshold", trace.get("specular_threshold", 0.0))
        for field, t in zip(("trace_rgb3", "trace_depth1", "trace_acc1", "trace_normal3", "trace_dist1",
                             "trace_aux2", "trace_mid32", "trace_wet1"), traced):
            setattr(view, field, _ptr(t))
    camera = maps = None
    if postprocess is not None:
        old_camera = out and out.camera
        camera_buf = take("camera", old_camera and old_camera["inverse_intrinsics"].view(-1)._base, (30,))
        pixel_rays = take("camera rays", old_camera and old_camera["rays"], (pixels, 3))
        maps = {name: take(name, out and out.maps and out.maps.get(name), (1, pixels, c))
                for name, c in zip(STANDARD_MAPS, STANDARD_MAP_CHANNELS)}
        view.fov_x = _finite("fov_x", postprocess["fov_x"])
        view.fov_y = _finite("fov_y", postprocess["fov_y"])
        view.depth_ratio = _finite("depth_ratio", postprocess.get("depth_ratio", 0.0))
        view.camera30 = _ptr(camera_buf)
        view.pixel_rays3 = _ptr(pixel_rays)
        for field, name in zip(("rgb_map3", "acc_map", "dpt_map", "norm_map3", "surf_norm_map3", "dist_map",
                                "spec_map", "rough_map"), STANDARD_MAPS):
            setattr(view, field, _ptr(maps[name]))
        camera = {"inverse_intrinsics": camera_buf[0:9].view(3, 3), "rotation": camera_buf[9:18].view(3, 3),
                  "origin": camera_buf[18:21], "normal_rotation": camera_buf[21:30].view(3, 3), "rays": pixel_rays}
    view.raster_begin_event = _event_handle(raster_begin_event)
    error = error_buffer()
    status = base_context.library.hs_b200_standard_view_v2(ctypes.byref(view), error, len(error))
    check_status(status, "hs_b200_standard_view_v2", error)
    return StandardViewOutputs(out_b, out_r, base_colors, refl_colors, rotation, normal, rays, origins, directions,
                               traced, fused, camera, maps)


def view_graph_stats(base_context: NativeRendererContext) -> dict[str, int]:
    """Graph replays of standard_view with ``base_context`` as its base
    context (hs_b200_view_graph_stats_v1): views captured, replayed, and
    replays rendered again directly because their pair count outgrew the
    capture."""
    values = [ctypes.c_uint64() for _ in range(3)]
    error = error_buffer()
    status = base_context.library.hs_b200_view_graph_stats_v1(base_context.handle,
                                                              *(ctypes.byref(v) for v in values), error, len(error))
    check_status(status, "hs_b200_view_graph_stats_v1", error)
    return dict(zip(("captures", "replays", "reruns"), (v.value for v in values)))


class FlashgsViewOutputs(NamedTuple):
    """Everything flashgs_view writes (the FlashGS counterpart of
    StandardViewOutputs; no raster colours are formed, the base call shades
    with SH and the reflection call takes the trace's or the given colours)."""
    base: FlashgsOutputs
    reflection: FlashgsOutputs
    reflection_rotation: torch.Tensor
    reflection_normal: torch.Tensor
    reflection_rays: torch.Tensor
    ray_origins: torch.Tensor | None
    ray_directions: torch.Tensor | None
    trace: TraceOutputs | None
    fused: dict[str, torch.Tensor]
    maps: dict[str, torch.Tensor] | None


FLASHGS_MAPS = ("rgb_map", "acc_map", "dpt_map", "norm_map", "surf_norm_map", "dist_map", "spec_map")
FLASHGS_MAP_CHANNELS = (3, 1, 1, 3, 3, 1, 1)


def flashgs_view(base: dict[str, Any], reflection: dict[str, Any], trace_group: dict[str, torch.Tensor],
                 world_view: torch.Tensor, full_proj: torch.Tensor, camera_center: torch.Tensor, *,
                 base_context: NativeRendererContext, reflection_context: NativeRendererContext,
                 trace: dict[str, Any] | None = None, postprocess: bool = False,
                 stream: int | None = None, raster_begin_event: torch.cuda.Event | None = None
                 ) -> FlashgsViewOutputs:
    """One view of the FlashGS session (render_hybridsplat_flashgs_view,
    renderer.py:344-446, with _flashgs_postprocess) in one call
    (hs_b200_flashgs_view_v2).

    ``base`` and ``reflection`` hold the arguments of flashgs_forward by name
    (no ``context``); the base call shades with SH (``use_sh=True``), the
    reflection call takes ``colors`` unless traced. ``trace_group`` is the
    standard-activated reflection group the session traces: ``means3d``,
    ``rotations_raw`` and, when traced, ``opacities``, ``scales``,
    ``rotations``. ``trace`` as in standard_view (``background``, ``shs``,
    ``others``, ``degree``, optional ``use_others``, ``max_trace_depth``,
    ``specular_threshold``); ``world_view``, ``full_proj`` and
    ``camera_center`` are the view's device camera. ``postprocess`` adds the
    FlashGS raw maps; ``raster_begin_event`` as in standard_view. Every output
    equals that of the same steps called one by one.
    """
    if base_context is reflection_context:
        raise ValueError("flashgs_view needs two distinct contexts")
    _check_tensor("world_view", world_view, (4, 4))
    _check_tensor("full_proj", full_proj, (4, 4))
    _check_tensor("camera_center", camera_center, (3,))
    device = world_view.device
    f = dict(dtype=torch.float32, device=device)
    nr = int(reflection["positions"].shape[0])
    _check_tensor("trace means3d", trace_group["means3d"], (nr, 3))
    _check_tensor("trace rotations_raw", trace_group["rotations_raw"], (nr, 4))
    traced = None
    reflection = dict(reflection)
    if trace is not None:
        traced = TraceOutputs(torch.empty((nr, 3), **f), torch.empty((nr, 1), **f), torch.empty((nr, 1), **f),
                              torch.empty((nr, 3), **f), torch.empty((nr, 1), **f), torch.empty((nr, 2), **f),
                              torch.empty((nr, 32), **f), torch.empty((nr, 1), **f))
        reflection["colors"] = traced.rgb
    named_b, out_b, hold_b = _flashgs_arguments(**dict(base, use_sh=True))
    named_r, out_r, hold_r = _flashgs_arguments(**dict(reflection, use_sh=False))
    whole = _rows_fields(None)
    rotation, normal, rays = torch.empty((nr, 3, 3), **f), torch.empty((nr, 3), **f), torch.empty((nr, 36), **f)
    origins = directions = None
    h, w = int(named_b["height"]), int(named_b["width"])
    fused = {k: torch.empty((h, w, 3), **f) for k in ("rgb_map", "dif_rgb_map", "ref_rgb_map")}
    view = native_runtime.FlashgsViewV2(
        struct_size=ctypes.sizeof(native_runtime.FlashgsViewV2),
        base=native_runtime.FlashgsCallV2(handle=base_context.handle, **named_b, **whole),
        reflection=native_runtime.FlashgsCallV2(handle=reflection_context.handle, **named_r, **whole),
        world_view4x4=_ptr(world_view), full_proj4x4=_ptr(full_proj), camera_center3=_ptr(camera_center),
        trace_means3d=_ptr(trace_group["means3d"]), trace_rotation_raw4=_ptr(trace_group["rotations_raw"]),
        reflection_rotation9=_ptr(rotation), reflection_normal3=_ptr(normal), reflection_rays36=_ptr(rays),
        fused_rgb3=_ptr(fused["rgb_map"]), diffuse_rgb3=_ptr(fused["dif_rgb_map"]),
        reflection_rgb_map3=_ptr(fused["ref_rgb_map"]), stream=stream)
    if trace is not None:
        shs = trace["shs"]
        coefficients = int(shs.shape[1])
        for name, t, shape in (("trace background", trace["background"], (3,)),
                               ("trace shs", shs, (nr, coefficients, 3)), ("trace others", trace["others"], (nr, 2)),
                               ("trace opacities", trace_group["opacities"], (nr, 1)),
                               ("trace scales", trace_group["scales"], (nr, 2)),
                               ("trace rotations", trace_group["rotations"], (nr, 4))):
            _check_tensor(name, t, shape)
        degree = trace["degree"]
        if isinstance(degree, bool) or not isinstance(degree, int) or degree not in range(4):
            raise ValueError("degree must be an integer in [0, 3]")
        depth = trace.get("max_trace_depth", 0)
        if depth not in (0, 1) or isinstance(depth, bool):
            raise ValueError("max_trace_depth must be 0 or 1")
        origins, directions = torch.empty((nr, 3), **f), torch.empty((nr, 3), **f)
        view.reflection_ray_origins3 = _ptr(origins)
        view.reflection_ray_directions3 = _ptr(directions)
        view.trace = 1
        view.trace_background3 = _ptr(trace["background"])
        view.trace_shs = _ptr(shs)
        view.trace_coefficients = coefficients
        view.trace_degree = degree
        view.trace_others2 = _ptr(trace["others"])
        view.trace_opacities = _ptr(trace_group["opacities"])
        view.trace_scales2 = _ptr(trace_group["scales"])
        view.trace_rotations4 = _ptr(trace_group["rotations"])
        view.use_others = int(bool(trace.get("use_others", True)))
        view.max_trace_depth = int(depth)
        view.specular_threshold = _finite("specular_threshold", trace.get("specular_threshold", 0.0))
        for field, t in zip(("trace_rgb3", "trace_depth1", "trace_acc1", "trace_normal3", "trace_dist1",
                             "trace_aux2", "trace_mid32", "trace_wet1"), traced):
            setattr(view, field, _ptr(t))
    maps = None
    if postprocess:
        maps = {n: torch.empty((1, h * w, c), **f) for n, c in zip(FLASHGS_MAPS, FLASHGS_MAP_CHANNELS)}
        view.postprocess = 1
        for field, name in zip(("rgb_map3", "acc_map", "dpt_map", "norm_map3", "surf_norm_map3", "dist_map",
                                "spec_map"), FLASHGS_MAPS):
            setattr(view, field, _ptr(maps[name]))
    view.raster_begin_event = _event_handle(raster_begin_event)
    error = error_buffer()
    status = base_context.library.hs_b200_flashgs_view_v2(ctypes.byref(view), error, len(error))
    del hold_b, hold_r
    check_status(status, "hs_b200_flashgs_view_v2", error)
    return FlashgsViewOutputs(out_b, out_r, rotation, normal, rays, origins, directions, traced, fused, maps)
