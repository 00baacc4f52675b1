"""ctypes binding of the HybridSplat rasterizer C ABI.

Mirrors the reference runtime ``jittor_hybridsplat/ops/native_runtime.py``
(`load_native_library` :164-423, `NativeRendererContext` :515-705): the same
struct layouts, ABI check (version 2), status handling and context methods.
Device synchronisation uses ``torch.cuda`` instead of Jittor, since PyTorch
owns device memory on this side of the boundary.

`bind_library(path)` applies the ABI signatures to any library that exports
them, so the same binding drives this package's sm_100a library and, in
tests, the reference build used as the parity oracle.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path
from typing import Any

HS_STATUS_OK = 0
HS_RASTERIZER_ABI_VERSION = 2
_ERROR_CAPACITY = 4096
_BUILD_INFO_CAPACITY = 8192

PACKAGE_DIR = Path(__file__).resolve().parent
LIBRARY_PATH = PACKAGE_DIR / "lib" / "libhybridsplat_rasterizer.so"


class NativeRasterizerError(RuntimeError):
    """Raised when a native entry point returns a non-OK HsStatus."""

    def __init__(self, message: str, status: int = -1):
        super().__init__(message)
        self.status = status


class _StatsBase(ctypes.Structure):
    def as_dict(self) -> dict[str, int]:
        return {name: int(getattr(self, name)) for name, _ in self._fields_}


class WorkspaceStatsV1(_StatsBase):
    _fields_ = [
        ("struct_size", ctypes.c_uint32),
        ("abi_version", ctypes.c_uint32),
        ("device", ctypes.c_int32),
        ("reserved", ctypes.c_uint32),
        ("geometry_bytes", ctypes.c_uint64),
        ("binning_bytes", ctypes.c_uint64),
        ("image_bytes", ctypes.c_uint64),
        ("current_bytes", ctypes.c_uint64),
        ("peak_bytes", ctypes.c_uint64),
        ("growth_count", ctypes.c_uint64),
    ]


class OptixWorkspaceStatsV1(_StatsBase):
    _fields_ = [
        ("struct_size", ctypes.c_uint32),
        ("abi_version", ctypes.c_uint32),
        ("device", ctypes.c_int32),
        ("scene_ready", ctypes.c_uint32),
        ("params_bytes", ctypes.c_uint64),
        ("gas_output_bytes", ctypes.c_uint64),
        ("gas_scratch_bytes", ctypes.c_uint64),
        ("dist3_bytes", ctypes.c_uint64),
        ("current_bytes", ctypes.c_uint64),
        ("peak_bytes", ctypes.c_uint64),
        ("growth_count", ctypes.c_uint64),
        ("scene_signature", ctypes.c_uint64),
        ("gas_build_count", ctypes.c_uint64),
        ("pipeline_create_count", ctypes.c_uint64),
    ]


class MathWorkspaceStatsV2(_StatsBase):
    _fields_ = [
        ("struct_size", ctypes.c_uint32),
        ("abi_version", ctypes.c_uint32),
        ("device", ctypes.c_int32),
        ("handles_ready", ctypes.c_uint32),
        ("workspace_bytes", ctypes.c_uint64),
        ("current_bytes", ctypes.c_uint64),
        ("peak_bytes", ctypes.c_uint64),
        ("growth_count", ctypes.c_uint64),
        ("handle_create_count", ctypes.c_uint64),
        ("camera_center_calls", ctypes.c_uint64),
        ("general_inverse_calls", ctypes.c_uint64),
        ("matmul_calls", ctypes.c_uint64),
        ("pixel_world_calls", ctypes.c_uint64),
    ]


class FlashgsWorkspaceStatsV1(_StatsBase):
    _fields_ = [
        ("struct_size", ctypes.c_uint32),
        ("abi_version", ctypes.c_uint32),
        ("device", ctypes.c_int32),
        ("initialized", ctypes.c_uint32),
        ("gaussian_capacity", ctypes.c_uint64),
        ("pair_capacity", ctypes.c_uint64),
        ("range_capacity", ctypes.c_uint64),
        ("output_pixel_capacity", ctypes.c_uint64),
        ("gaussian_bytes", ctypes.c_uint64),
        ("pair_bytes", ctypes.c_uint64),
        ("cub_bytes", ctypes.c_uint64),
        ("ranges_bytes", ctypes.c_uint64),
        ("output_bytes", ctypes.c_uint64),
        ("current_bytes", ctypes.c_uint64),
        ("peak_bytes", ctypes.c_uint64),
        ("growth_count", ctypes.c_uint64),
        ("overflow_retry_count", ctypes.c_uint64),
        ("forward_calls", ctypes.c_uint64),
        ("last_point_count", ctypes.c_uint64),
        ("last_num_rendered", ctypes.c_uint64),
        ("last_tile_count", ctypes.c_uint64),
    ]


_V = ctypes.c_void_p
_U64 = ctypes.c_uint64
_U32 = ctypes.c_uint32
_I32 = ctypes.c_int32
_F = ctypes.c_float
_ERR = [ctypes.c_char_p, _U64]

# Argument lists of every exported symbol (include/hybridsplat_rasterizer_c_api.h).
# Device and host tensors are passed as raw addresses (c_void_p).
SIGNATURES: dict[str, tuple[Any, list[Any]]] = {
    "hs_rasterizer_abi_version": (_U32, []),
    "hs_rasterizer_build_info": (_I32, [ctypes.c_char_p, _U64]),
    "hs_rasterizer_create": (_I32, [_I32, ctypes.POINTER(ctypes.c_void_p), *_ERR]),
    "hs_rasterizer_synchronize": (_I32, [_V, *_ERR]),
    "hs_rasterizer_workspace_stats": (_I32, [_V, ctypes.POINTER(WorkspaceStatsV1), *_ERR]),
    "hs_rasterizer_release_workspace": (_I32, [_V, *_ERR]),
    "hs_rasterizer_math_workspace_stats_v2": (_I32, [_V, ctypes.POINTER(MathWorkspaceStatsV2), *_ERR]),
    "hs_rasterizer_destroy": (_I32, [_V, *_ERR]),
    "hs_flashgs_forward_f32_v1": (
        _I32,
        [_V, _U64, _I32, _I32, _V, _V, _V, _I32, _V, _V, _V, _F, _V, _V, _V, _V, _V, _F, _F, _F,
         _F, _V, _U64, _V, _V, _V, _V, _V, _V, _V, _V, *_ERR],
    ),
    "hs_flashgs_workspace_stats_v1": (_I32, [_V, ctypes.POINTER(FlashgsWorkspaceStatsV1), *_ERR]),
    "hs_flashgs_prepare_npz_host_f32_v1": (_I32, [_U64, _V, _V, _V, _V, _V, _V, _V, _V, _V, _V, _V, *_ERR]),
    "hs_flashgs_debug_copy_v1": (_I32, [_V, _U64, _U64, _U64, _V, _V, _V, _V, _V, _V, _V, _V, _V, _V, _V, *_ERR]),
    "hs_rasterizer_forward_f32_v1": (
        _I32,
        [_V, _U64, _V, _I32, _I32, _V, _V, _V, _V, _F, _V, _V, _V, _V, _F, _F, _I32, _V, _V, _V, _V,
         _V, *_ERR],
    ),
    "hs_optix_build_scene_v1": (_I32, [_V, _V, _U64, _V, _U64, _U64, _I32, _V, *_ERR]),
    "hs_optix_trace_f32_v1": (
        _I32,
        [_V, _U64, _V, _V, _V, _V, _V, _U32, _U32, _V, _V, _V, _F, _V, _V, _V, _V, _I32, _I32, _F,
         _I32, _V, _V, _V, _V, _V, _V, _V, _V, *_ERR],
    ),
    "hs_optix_workspace_stats_v1": (_I32, [_V, ctypes.POINTER(OptixWorkspaceStatsV1), *_ERR]),
    "hs_optix_release_scene_v1": (_I32, [_V, *_ERR]),
    "hs_rasterizer_precise_exp_f32_v1": (_I32, [_V, _V, _U64, *_ERR]),
    "hs_rasterizer_precise_sigmoid_f32_v1": (_I32, [_V, _V, _U64, *_ERR]),
    "hs_rasterizer_precise_normalize4_f32_v1": (_I32, [_V, _V, _U64, *_ERR]),
    "hs_rasterizer_precise_fuse_maps_f32_v1": (_I32, [_V, _V, _V, _V, _V, _V, _U64, *_ERR]),
    "hs_rasterizer_precise_sh_to_rgb_f32_v1": (_I32, [_V, _V, _U64, _U32, _U32, _V, *_ERR]),
    "hs_rasterizer_precise_direction_f32_v1": (_I32, [_V, _V, _U64, _V, *_ERR]),
    "hs_rasterizer_precise_camera_center_f32_v2": (_I32, [_V, _V, _V, _V, *_ERR]),
    "hs_rasterizer_precise_general_inverse_f32_v2": (_I32, [_V, _V, _U32, _V, *_ERR]),
    "hs_rasterizer_precise_matmul_nt_n3k3_f32_v2": (_I32, [_V, _V, _V, _U64, _V, *_ERR]),
    "hs_rasterizer_precise_pixel_world_f32_v2": (_I32, [_V, _V, _V, _U64, _V, *_ERR]),
    "hs_rasterizer_precise_disk_rotation_f32_v1": (_I32, [_V, _U64, _V, *_ERR]),
    "hs_rasterizer_precise_reflection_prefix_f32_v1": (_I32, [_V, _U64, _V, *_ERR]),
    "hs_rasterizer_precise_reflection_suffix_f32_v1": (_I32, [_V, _V, _V, _U64, _V, *_ERR]),
}

# Extensions of this library (include/hybridsplat_b200_ext.h); the reference
# library does not export them, so they are bound only where present.
class FlashgsCallV2(ctypes.Structure):
    """HsB200FlashgsCallV2 (include/hybridsplat_b200_ext.h)."""
    _fields_ = [
        ("handle", ctypes.c_void_p), ("point_count", ctypes.c_uint64), ("width", ctypes.c_int32),
        ("height", ctypes.c_int32), ("positions3", ctypes.c_void_p), ("shs48", ctypes.c_void_p),
        ("colors3", ctypes.c_void_p), ("use_sh", ctypes.c_int32), ("scale_modifier", ctypes.c_float),
        ("opacities1", ctypes.c_void_p), ("covariance6", ctypes.c_void_p), ("scales2", ctypes.c_void_p),
        ("rotations4", ctypes.c_void_p), ("specular1", ctypes.c_void_p), ("roughness1", ctypes.c_void_p),
        ("camera_position3", ctypes.c_void_p), ("camera_rotation9", ctypes.c_void_p),
        ("focal_x", ctypes.c_float), ("focal_y", ctypes.c_float), ("z_far", ctypes.c_float),
        ("z_near", ctypes.c_float), ("background3", ctypes.c_void_p), ("initial_pair_capacity", ctypes.c_uint64),
        ("output_color3", ctypes.c_void_p), ("output_other2", ctypes.c_void_p), ("output_depth1", ctypes.c_void_p),
        ("output_alpha1", ctypes.c_void_p), ("output_normal3", ctypes.c_void_p),
        ("output_median_depth1", ctypes.c_void_p), ("output_distortion1", ctypes.c_void_p),
        ("output_num_rendered", ctypes.c_void_p), ("tile_row_begin", ctypes.c_uint32),
        ("tile_row_end", ctypes.c_uint32),
    ]


class RasterizerCallV2(ctypes.Structure):
    """HsB200RasterizerCallV2 (include/hybridsplat_b200_ext.h)."""
    _fields_ = [
        ("handle", ctypes.c_void_p), ("point_count", ctypes.c_uint64), ("background5", ctypes.c_void_p),
        ("width", ctypes.c_int32), ("height", ctypes.c_int32), ("means3d", ctypes.c_void_p),
        ("colors5", ctypes.c_void_p), ("opacities", ctypes.c_void_p), ("scales2", ctypes.c_void_p),
        ("scale_modifier", ctypes.c_float), ("prefiltered", ctypes.c_int32), ("rotations4", ctypes.c_void_p),
        ("viewmatrix4x4", ctypes.c_void_p), ("projmatrix4x4", ctypes.c_void_p),
        ("camera_position3", ctypes.c_void_p), ("tan_fovx", ctypes.c_float), ("tan_fovy", ctypes.c_float),
        ("output_color5", ctypes.c_void_p), ("output_aux7", ctypes.c_void_p), ("output_weight", ctypes.c_void_p),
        ("output_radii", ctypes.c_void_p), ("output_rendered", ctypes.c_void_p),
        ("tile_row_begin", ctypes.c_uint32), ("tile_row_end", ctypes.c_uint32),
    ]


class StandardGroupV2(ctypes.Structure):
    """HsB200StandardGroupV2 (include/hybridsplat_b200_ext.h)."""
    _fields_ = [
        ("count", ctypes.c_uint64), ("means3d", ctypes.c_void_p), ("opacities", ctypes.c_void_p),
        ("scales2", ctypes.c_void_p), ("rotations4", ctypes.c_void_p), ("specular", ctypes.c_void_p),
        ("roughness", ctypes.c_void_p), ("background5", ctypes.c_void_p), ("colors5", ctypes.c_void_p),
        ("output_color5", ctypes.c_void_p), ("output_aux7", ctypes.c_void_p), ("output_weight", ctypes.c_void_p),
        ("output_radii", ctypes.c_void_p), ("output_rendered", ctypes.c_void_p),
    ]


class StandardViewV2(ctypes.Structure):
    """HsB200StandardViewV2 (include/hybridsplat_b200_ext.h)."""
    _fields_ = [
        ("struct_size", ctypes.c_uint32), ("base_handle", ctypes.c_void_p), ("reflection_handle", ctypes.c_void_p),
        ("width", ctypes.c_int32), ("height", ctypes.c_int32), ("tan_fovx", ctypes.c_float),
        ("tan_fovy", ctypes.c_float), ("fov_x", ctypes.c_double), ("fov_y", ctypes.c_double),
        ("viewmatrix4x4", ctypes.c_void_p), ("projmatrix4x4", ctypes.c_void_p),
        ("camera_position3", ctypes.c_void_p), ("base", StandardGroupV2), ("reflection", StandardGroupV2),
        ("base_sh", ctypes.c_void_p), ("sh_coefficients", ctypes.c_uint32), ("sh_degree", ctypes.c_uint32),
        ("reflection_rotation_raw4", ctypes.c_void_p), ("reflection_rotation9", ctypes.c_void_p),
        ("reflection_normal3", ctypes.c_void_p), ("reflection_rays36", ctypes.c_void_p),
        ("reflection_ray_origins3", ctypes.c_void_p), ("reflection_ray_directions3", ctypes.c_void_p),
        ("reflection_rgb3", ctypes.c_void_p), ("trace", ctypes.c_int32), ("trace_background3", ctypes.c_void_p),
        ("reflection_shs", ctypes.c_void_p), ("trace_coefficients", ctypes.c_uint32),
        ("trace_degree", ctypes.c_uint32), ("reflection_others2", ctypes.c_void_p), ("use_others", ctypes.c_int32),
        ("max_trace_depth", ctypes.c_int32), ("specular_threshold", ctypes.c_float),
        ("trace_rgb3", ctypes.c_void_p), ("trace_depth1", ctypes.c_void_p), ("trace_acc1", ctypes.c_void_p),
        ("trace_normal3", ctypes.c_void_p), ("trace_dist1", ctypes.c_void_p), ("trace_aux2", ctypes.c_void_p),
        ("trace_mid32", ctypes.c_void_p), ("trace_wet1", ctypes.c_void_p), ("fused_rgb3", ctypes.c_void_p),
        ("diffuse_rgb3", ctypes.c_void_p), ("reflection_rgb_map3", ctypes.c_void_p),
        ("depth_ratio", ctypes.c_double), ("camera30", ctypes.c_void_p), ("pixel_rays3", ctypes.c_void_p),
        ("rgb_map3", ctypes.c_void_p), ("acc_map", ctypes.c_void_p), ("dpt_map", ctypes.c_void_p),
        ("norm_map3", ctypes.c_void_p), ("surf_norm_map3", ctypes.c_void_p), ("dist_map", ctypes.c_void_p),
        ("spec_map", ctypes.c_void_p), ("rough_map", ctypes.c_void_p), ("raster_begin_event", ctypes.c_void_p),
        ("stream", ctypes.c_void_p),
    ]


class FlashgsViewV2(ctypes.Structure):
    """HsB200FlashgsViewV2 (include/hybridsplat_b200_ext.h)."""
    _fields_ = [
        ("struct_size", ctypes.c_uint32), ("base", FlashgsCallV2), ("reflection", FlashgsCallV2),
        ("world_view4x4", ctypes.c_void_p), ("full_proj4x4", ctypes.c_void_p), ("camera_center3", ctypes.c_void_p),
        ("trace_means3d", ctypes.c_void_p), ("trace_rotation_raw4", ctypes.c_void_p),
        ("reflection_rotation9", ctypes.c_void_p), ("reflection_normal3", ctypes.c_void_p),
        ("reflection_rays36", ctypes.c_void_p), ("reflection_ray_origins3", ctypes.c_void_p),
        ("reflection_ray_directions3", ctypes.c_void_p), ("trace", ctypes.c_int32),
        ("trace_background3", ctypes.c_void_p), ("trace_shs", ctypes.c_void_p),
        ("trace_coefficients", ctypes.c_uint32), ("trace_degree", ctypes.c_uint32),
        ("trace_others2", ctypes.c_void_p), ("trace_opacities", ctypes.c_void_p), ("trace_scales2", ctypes.c_void_p),
        ("trace_rotations4", ctypes.c_void_p), ("use_others", ctypes.c_int32), ("max_trace_depth", ctypes.c_int32),
        ("specular_threshold", ctypes.c_float), ("trace_rgb3", ctypes.c_void_p), ("trace_depth1", ctypes.c_void_p),
        ("trace_acc1", ctypes.c_void_p), ("trace_normal3", ctypes.c_void_p), ("trace_dist1", ctypes.c_void_p),
        ("trace_aux2", ctypes.c_void_p), ("trace_mid32", ctypes.c_void_p), ("trace_wet1", ctypes.c_void_p),
        ("fused_rgb3", ctypes.c_void_p), ("diffuse_rgb3", ctypes.c_void_p), ("reflection_rgb_map3", ctypes.c_void_p),
        ("postprocess", ctypes.c_int32), ("rgb_map3", ctypes.c_void_p), ("acc_map", ctypes.c_void_p),
        ("dpt_map", ctypes.c_void_p), ("norm_map3", ctypes.c_void_p), ("surf_norm_map3", ctypes.c_void_p),
        ("dist_map", ctypes.c_void_p), ("spec_map", ctypes.c_void_p), ("raster_begin_event", ctypes.c_void_p),
        ("stream", ctypes.c_void_p),
    ]


EXTENSION_SIGNATURES: dict[str, tuple[Any, list[Any]]] = {
    "hs_b200_precise_sh_colors5_f32_v1": (_I32, [_V, _U32, _U32, _V, _V, _V, _V, _U64, _V, *_ERR]),
    "hs_b200_precise_fuse_maps_planar_f32_v1": (_I32, [_V, _V, _V, _V, _V, _V, _U64, *_ERR]),
    "hs_b200_standard_debug_copy_v1": (_I32, [_V, _U64, _V, _V, _V, *_ERR]),
    "hs_b200_postprocess_camera_f32_v1": (_I32, [_V, _I32, _I32, ctypes.c_double, ctypes.c_double, _V, _V, _V, _V,
                                                   *_ERR]),
    "hs_b200_pixel_rays_f32_v1": (_I32, [_V, _I32, _I32, _V, _V, _V, _V, *_ERR]),
    "hs_b200_standard_postprocess_f32_v1": (_I32, [_I32, _I32, _V, _V, _V, _V, _V, ctypes.c_double,
                                                   _V, _V, _V, _V, _V, _V, _V, _V, *_ERR]),
    "hs_b200_flashgs_postprocess_f32_v1": (_I32, [_I32, _I32, _V, _V, _V, _V, _V, _V, _V, _V, _V, _V,
                                                  _V, _V, _V, *_ERR]),
    "hs_b200_flashgs_forward_many_v2": (_I32, [ctypes.POINTER(FlashgsCallV2), _U32, _V, *_ERR]),
    "hs_b200_rasterizer_forward_many_v2": (_I32, [ctypes.POINTER(RasterizerCallV2), _U32, _V, *_ERR]),
    "hs_b200_standard_view_v2": (_I32, [ctypes.POINTER(StandardViewV2), *_ERR]),
    "hs_b200_flashgs_view_v2": (_I32, [ctypes.POINTER(FlashgsViewV2), *_ERR]),
    "hs_b200_test_stall_lookback_v1": (_I32, [_V, _U32, *_ERR]),
    "hs_b200_test_pair_ops_v1": (_I32, [_V, _V, _V, _V, _U64, _V, *_ERR]),
    "hs_b200_view_graph_stats_v1": (_I32, [_V, _V, _V, _V, *_ERR]),
    "hs_b200_comm_unique_id_v1": (_I32, [_V, *_ERR]),
    "hs_b200_comm_create_v1": (_I32, [_I32, _I32, _I32, _V, ctypes.c_double, ctypes.POINTER(ctypes.c_void_p),
                                      *_ERR]),
    "hs_b200_comm_broadcast_v1": (_I32, [_V, _V, _U64, _I32, _V, *_ERR]),
    "hs_b200_comm_allreduce_max_f64_v1": (_I32, [_V, _V, _V, _U32, *_ERR]),
    "hs_b200_comm_barrier_v1": (_I32, [_V, *_ERR]),
    "hs_b200_comm_destroy_v1": (_I32, [_V, *_ERR]),
    "hs_b200_stage_timing_enable_v1": (_I32, [_V, _I32, *_ERR]),
    "hs_b200_stage_timing_read_v1": (_I32, [_V, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(_U64), *_ERR]),
    "hs_b200_flashgs_forward_rows_f32_v1": (
        _I32,
        [_V, _U32, _U32, _U64, _I32, _I32, _V, _V, _V, _I32, _V, _V, _V, _F, _V, _V, _V, _V, _V, _F, _F, _F,
         _F, _V, _U64, _V, _V, _V, _V, _V, _V, _V, _V, *_ERR],
    ),
    "hs_b200_rasterizer_forward_rows_f32_v1": (
        _I32,
        [_V, _U32, _U32, _U64, _V, _I32, _I32, _V, _V, _V, _V, _F, _V, _V, _V, _V, _F, _F, _I32, _V, _V, _V,
         _V, _V, *_ERR],
    ),
    "hs_b200_rasterizer_forward_noalloc_f32_v1": (
        _I32,
        [_I32, _U64, _V, _I32, _I32, _V, _V, _V, _V, _F, _V, _V, _V, _V, _F, _F, _I32, _V, _V, _V, _V,
         _V, *_ERR],
    ),
}

# Entry points that the reference's OptiX-free oracle build does not export.
OPTIX_SYMBOLS = {
    "hs_optix_build_scene_v1",
    "hs_optix_trace_f32_v1",
    "hs_optix_workspace_stats_v1",
    "hs_optix_release_scene_v1",
}


def error_buffer() -> ctypes.Array[ctypes.c_char]:
    return ctypes.create_string_buffer(_ERROR_CAPACITY)


def check_status(status: int, operation: str, error: ctypes.Array[ctypes.c_char]) -> None:
    if status != HS_STATUS_OK:
        detail = error.value.decode("utf-8", errors="replace")
        raise NativeRasterizerError(f"{operation} failed with native status {status}: {detail}", status)


def bind_library(path: Path | str, *, require_optix: bool = True) -> ctypes.CDLL:
    """Loads a library exporting the C ABI and sets every signature.

    Raises NativeRasterizerError if the file is missing, a symbol is absent
    or the ABI version differs from 2.
    """
    path = Path(path)
    if not path.is_file():
        raise NativeRasterizerError(
            f"native rasterizer library not found at {path}; build it with "
            "`python -m hybridsplat_jittor_render_b200.build`"
        )
    library = ctypes.CDLL(str(path), mode=os.RTLD_LOCAL | os.RTLD_NOW)
    for name, (restype, argtypes) in SIGNATURES.items():
        if not require_optix and name in OPTIX_SYMBOLS:
            continue
        try:
            function = getattr(library, name)
        except AttributeError as exc:
            raise NativeRasterizerError(f"{path} does not export {name}") from exc
        function.restype = restype
        function.argtypes = argtypes
    for name, (restype, argtypes) in EXTENSION_SIGNATURES.items():
        if hasattr(library, name):
            getattr(library, name).restype = restype
            getattr(library, name).argtypes = argtypes
    version = int(library.hs_rasterizer_abi_version())
    if version != HS_RASTERIZER_ABI_VERSION:
        raise NativeRasterizerError(
            f"{path} has ABI version {version}, expected {HS_RASTERIZER_ABI_VERSION}"
        )
    return library


_LIBRARY: ctypes.CDLL | None = None
_LOAD_LOCK = threading.Lock()


def load_native_library() -> ctypes.CDLL:
    """The sm_100a library of this package (loaded once, never a fallback)."""
    global _LIBRARY
    with _LOAD_LOCK:
        if _LIBRARY is None:
            _LIBRARY = bind_library(LIBRARY_PATH)
        return _LIBRARY


def _torch_synchronize(device: int) -> None:
    try:
        import torch
    except ImportError:  # pragma: no cover - torch is a hard dependency on GPU hosts
        return
    if torch.cuda.is_available():
        torch.cuda.synchronize(device)


class NativeRendererContext:
    """Owns one native context (HsRasterizerHandle) on one CUDA device.

    Same surface as the reference NativeRendererContext
    (native_runtime.py:515-705). `library` selects the shared library; the
    default is this package's sm_100a build.
    """

    def __init__(self, device: int = 0, *, library: ctypes.CDLL | None = None):
        self._library = library if library is not None else load_native_library()
        self._device = int(device)
        self._handle = ctypes.c_void_p()
        error = error_buffer()
        status = self._library.hs_rasterizer_create(self._device, ctypes.byref(self._handle), error, len(error))
        check_status(status, "hs_rasterizer_create", error)

    @property
    def library(self) -> ctypes.CDLL:
        return self._library

    @property
    def device(self) -> int:
        return self._device

    @property
    def handle(self) -> ctypes.c_void_p:
        if self._handle.value is None:
            raise NativeRasterizerError("native rasterizer context is closed")
        return self._handle

    @property
    def handle_value(self) -> int:
        return int(self.handle.value)

    @property
    def build_info(self) -> str:
        output = ctypes.create_string_buffer(_BUILD_INFO_CAPACITY)
        status = self._library.hs_rasterizer_build_info(output, len(output))
        check_status(status, "hs_rasterizer_build_info", output)
        return output.value.decode("utf-8")

    def synchronize(self) -> None:
        _torch_synchronize(self._device)
        error = error_buffer()
        status = self._library.hs_rasterizer_synchronize(self.handle, error, len(error))
        check_status(status, "hs_rasterizer_synchronize", error)

    def _stats(self, symbol: str, struct_type: type[_StatsBase]) -> dict[str, int]:
        stats = struct_type()
        stats.struct_size = ctypes.sizeof(struct_type)
        stats.abi_version = HS_RASTERIZER_ABI_VERSION
        error = error_buffer()
        status = getattr(self._library, symbol)(self.handle, ctypes.byref(stats), error, len(error))
        check_status(status, symbol, error)
        return stats.as_dict()

    def workspace_stats(self) -> dict[str, int]:
        return self._stats("hs_rasterizer_workspace_stats", WorkspaceStatsV1)

    def math_workspace_stats(self) -> dict[str, int]:
        return self._stats("hs_rasterizer_math_workspace_stats_v2", MathWorkspaceStatsV2)

    def optix_workspace_stats(self) -> dict[str, int]:
        return self._stats("hs_optix_workspace_stats_v1", OptixWorkspaceStatsV1)

    def flashgs_workspace_stats(self) -> dict[str, int]:
        return self._stats("hs_flashgs_workspace_stats_v1", FlashgsWorkspaceStatsV1)

    def stage_timing(self, enable: bool) -> None:
        """Turns per-stage device timing of the raster calls on or off
        (library extension; absent from the reference library)."""
        error = error_buffer()
        status = self._library.hs_b200_stage_timing_enable_v1(self.handle, int(bool(enable)), error, len(error))
        check_status(status, "hs_b200_stage_timing_enable_v1", error)

    def read_stage_timing(self) -> dict[str, float]:
        """Summed preprocess / binning / blending ms of the raster calls
        timed since the previous read, and their count."""
        ms = (ctypes.c_double * 3)()
        calls = _U64(0)
        error = error_buffer()
        status = self._library.hs_b200_stage_timing_read_v1(self.handle, ms, ctypes.byref(calls), error,
                                                            len(error))
        check_status(status, "hs_b200_stage_timing_read_v1", error)
        return {"preprocess_ms": ms[0], "binning_ms": ms[1], "blend_ms": ms[2], "calls": int(calls.value)}

    def stall_next_sort(self, tile: int) -> None:
        """Test hook: the next raster call's depth sort runs with sort tile
        `tile` of its first pass never publishing its look-back status, so the
        bounded waits behind it run out and that call fails
        (hs_b200_test_stall_lookback_v1)."""
        error = error_buffer()
        status = self._library.hs_b200_test_stall_lookback_v1(self.handle, int(tile), error, len(error))
        check_status(status, "hs_b200_test_stall_lookback_v1", error)

    def release_workspace(self) -> None:
        _torch_synchronize(self._device)
        error = error_buffer()
        status = self._library.hs_rasterizer_release_workspace(self.handle, error, len(error))
        check_status(status, "hs_rasterizer_release_workspace", error)

    def release_optix_scene(self) -> None:
        error = error_buffer()
        status = self._library.hs_optix_release_scene_v1(self.handle, error, len(error))
        check_status(status, "hs_optix_release_scene_v1", error)

    def flashgs_debug_snapshot(self) -> dict[str, Any]:
        """Host copies of the last FlashGS preprocess, sorted pairs and ranges."""
        import numpy as np

        _torch_synchronize(self._device)
        stats = self.flashgs_workspace_stats()
        points, pairs, tiles = stats["last_point_count"], stats["last_num_rendered"], stats["last_tile_count"]
        arrays = {
            "points_xy": np.empty((points, 2), np.float32),
            "rgb": np.empty((points, 3), np.float32),
            "other_features": np.empty((points, 2), np.float32),
            "conic_opacity": np.empty((points, 4), np.float32),
            "normal_opacity": np.empty((points, 4), np.float32),
            "Tu": np.empty((points, 3), np.float32),
            "Tv": np.empty((points, 3), np.float32),
            "Tw": np.empty((points, 3), np.float32),
            "sorted_keys": np.empty(pairs, np.uint64),
            "sorted_values": np.empty(pairs, np.uint32),
            "tile_ranges": np.empty((tiles, 2), np.int32),
        }
        error = error_buffer()
        names = ("points_xy", "rgb", "other_features", "conic_opacity", "normal_opacity", "Tu", "Tv", "Tw",
                 "sorted_keys", "sorted_values", "tile_ranges")
        status = self._library.hs_flashgs_debug_copy_v1(
            self.handle, points, pairs, tiles, *[arrays[n].ctypes.data for n in names], error, len(error)
        )
        check_status(status, "hs_flashgs_debug_copy_v1", error)
        return arrays

    def standard_debug_snapshot(self, point_count: int) -> dict[str, Any]:
        """Host copies of the last standard forward's per-Gaussian blend state
        (centre, Tu|Tv|Tw rows, normal|opacity) for its `point_count` Gaussians;
        rows of Gaussians with radius 0 are unspecified."""
        import numpy as np

        _torch_synchronize(self._device)
        arrays = {"points_xy": np.empty((point_count, 2), np.float32),
                  "transmats": np.empty((point_count, 9), np.float32),
                  "normal_opacity": np.empty((point_count, 4), np.float32)}
        error = error_buffer()
        status = self._library.hs_b200_standard_debug_copy_v1(
            self.handle, point_count, *[a.ctypes.data for a in arrays.values()], error, len(error))
        check_status(status, "hs_b200_standard_debug_copy_v1", error)
        return arrays

    def close(self) -> None:
        if self._handle.value is None:
            return
        _torch_synchronize(self._device)
        error = error_buffer()
        status = self._library.hs_rasterizer_destroy(self._handle, error, len(error))
        check_status(status, "hs_rasterizer_destroy", error)
        self._handle = ctypes.c_void_p()

    def __enter__(self) -> "NativeRendererContext":
        return self

    def __exit__(self, *exc: Any) -> None:
        self.close()

    def __del__(self) -> None:  # pragma: no cover - best effort at interpreter exit
        try:
            if self._handle.value is not None:
                error = error_buffer()
                self._library.hs_rasterizer_destroy(self._handle, error, len(error))
                self._handle = ctypes.c_void_p()
        except Exception:
            pass
