"""C-ABI surface checks that need no GPU.

* the library loads, reports ABI 2 and exports every symbol declared in
  include/*.h;
* argument validation (status codes and messages) matches the reference
  library for invalid calls that are rejected before any CUDA work
  (reference rasterizer/c_api.cpp:792-884, 1037-1094, 1136-1910);
* the host FlashGS activation is bit-identical to the reference's own build.
"""

from __future__ import annotations

import ctypes
import json
import re

import numpy as np
import pytest

from conftest import REF_LIBRARY, REF_PREPARE, REPO
from hybridsplat_jittor_render_b200 import native_runtime as nr
from hybridsplat_jittor_render_b200 import ops

HEADER = REPO / "include" / "hybridsplat_rasterizer_c_api.h"


def declared_symbols(header=None) -> list[str]:
    """Entry points declared by one header, or by every header in include/."""
    files = [header] if header is not None else sorted((REPO / "include").glob("*.h"))
    names = []
    for f in files:
        names += re.findall(r"HS_API\s+[a-z0-9_]+\s+(hs_[a-z0-9_]+)\s*\(", f.read_text())
    return names


@pytest.fixture(scope="module")
def lib():
    return nr.load_native_library()


@pytest.fixture(scope="module")
def ref():
    if not REF_LIBRARY.exists():
        pytest.skip("reference build absent")
    return nr.bind_library(REF_LIBRARY, require_optix=False)


def test_exports_every_declared_symbol(lib):
    symbols = declared_symbols()
    assert len(declared_symbols(HEADER)) >= 30
    for name in symbols:
        assert hasattr(lib, name), name
    assert set(nr.SIGNATURES) == set(declared_symbols(HEADER))
    assert set(nr.SIGNATURES) | set(nr.EXTENSION_SIGNATURES) == set(symbols)


def test_abi_version_and_build_info(lib):
    assert lib.hs_rasterizer_abi_version() == 2
    buf = ctypes.create_string_buffer(4096)
    assert lib.hs_rasterizer_build_info(buf, len(buf)) == 0
    info = json.loads(buf.value.decode())
    assert info["abi"] == 2 and info["arch"] == "sm_100a"
    small = ctypes.create_string_buffer(8)
    assert lib.hs_rasterizer_build_info(small, len(small)) == 3  # RANGE_ERROR, truncated
    assert len(small.value) == 7
    assert lib.hs_rasterizer_build_info(None, 0) == 1


def _flashgs_call(library, *, handle=None, width=64, height=48, count=0, use_sh=1, capacity=1024,
                  focal=100.0, znear=0.01, zfar=100.0, scale=1.0, camera_ok=True, outputs=True):
    pos = (ctypes.c_float * 3)(0.0, 0.0, 0.0)
    rot = (ctypes.c_float * 9)(1, 0, 0, 0, 1, 0, 0, 0, 1)
    if not camera_ok:
        rot[4] = float("nan")
    bg = (ctypes.c_float * 3)(0, 0, 0)
    dummy = ctypes.c_void_p(16)  # never dereferenced: validation fails first
    outs = [dummy] * 8 if outputs else [None] * 8
    err = ctypes.create_string_buffer(512)
    status = library.hs_flashgs_forward_f32_v1(
        handle, count, width, height, None, None, None, use_sh, None, None, None, scale, None, None, None,
        ctypes.addressof(pos), ctypes.addressof(rot), focal, focal, zfar, znear, ctypes.addressof(bg), capacity,
        *outs, err, len(err))
    return status, err.value.decode()


@pytest.mark.parametrize("kwargs", [
    dict(handle=None),
    dict(handle=ctypes.c_void_p(16), outputs=False),
    dict(handle=ctypes.c_void_p(16), width=0),
    dict(handle=ctypes.c_void_p(16), height=-3),
    dict(handle=ctypes.c_void_p(16), use_sh=2),
    dict(handle=ctypes.c_void_p(16), capacity=0),
    dict(handle=ctypes.c_void_p(16), capacity=1 << 40),
    dict(handle=ctypes.c_void_p(16), focal=-1.0),
    dict(handle=ctypes.c_void_p(16), znear=0.0),
    dict(handle=ctypes.c_void_p(16), zfar=0.005),
    dict(handle=ctypes.c_void_p(16), scale=float("inf")),
    dict(handle=ctypes.c_void_p(16), camera_ok=False),
    dict(handle=ctypes.c_void_p(16), count=5),  # non-empty with null inputs
    dict(handle=ctypes.c_void_p(16), count=1 << 33),
])
def test_flashgs_validation_matches_reference(lib, ref, kwargs):
    assert _flashgs_call(lib, **kwargs) == _flashgs_call(ref, **kwargs)


def test_error_buffer_contract(lib, ref):
    for library in (lib, ref):
        assert library.hs_rasterizer_synchronize(None, None, 16) == 1
    status, message = _flashgs_call(lib, handle=None)
    assert status == 1 and message == "FlashGS received a null required handle or buffer"


def _raster_call(library, *, handle=ctypes.c_void_p(16), width=64, height=48, count=0, tanx=0.5, prefiltered=0,
                 bg=True):
    dummy = ctypes.c_void_p(16)
    err = ctypes.create_string_buffer(512)
    status = library.hs_rasterizer_forward_f32_v1(
        handle, count, dummy if bg else None, width, height, None, None, None, None, 1.0, None, None, None, None,
        tanx, 0.5, prefiltered, dummy, dummy, None, None, dummy, err, len(err))
    return status, err.value.decode()


@pytest.mark.parametrize("kwargs", [
    dict(handle=None), dict(bg=False), dict(width=0), dict(tanx=0.0), dict(tanx=float("nan")),
    dict(prefiltered=3), dict(count=4),
])
def test_rasterizer_validation_matches_reference(lib, ref, kwargs):
    assert _raster_call(lib, **kwargs) == _raster_call(ref, **kwargs)


@pytest.mark.parametrize("symbol,args", [
    ("hs_rasterizer_precise_exp_f32_v1", (None, None, 0)),
    ("hs_rasterizer_precise_exp_f32_v1", (None, None, 10)),
    ("hs_rasterizer_precise_sigmoid_f32_v1", (None, None, 10)),
    ("hs_rasterizer_precise_normalize4_f32_v1", (None, None, 10)),
    ("hs_rasterizer_precise_fuse_maps_f32_v1", (None, None, None, None, None, None, 10)),
    ("hs_rasterizer_precise_sh_to_rgb_f32_v1", (None, None, 10, 16, 4, None)),
    ("hs_rasterizer_precise_sh_to_rgb_f32_v1", (None, None, 10, 8, 3, None)),
    ("hs_rasterizer_precise_sh_to_rgb_f32_v1", (None, None, 0, 16, 3, None)),
    ("hs_rasterizer_precise_direction_f32_v1", (None, None, 10, None)),
    ("hs_rasterizer_precise_disk_rotation_f32_v1", (None, 10, None)),
    ("hs_rasterizer_precise_reflection_prefix_f32_v1", (None, 10, None)),
    ("hs_rasterizer_precise_reflection_suffix_f32_v1", (None, None, None, 10, None)),
    ("hs_rasterizer_precise_general_inverse_f32_v2", (None, None, 5, None)),
    ("hs_rasterizer_precise_matmul_nt_n3k3_f32_v2", (None, None, None, 0, None)),
    ("hs_rasterizer_precise_pixel_world_f32_v2", (None, None, None, 0, None)),
])
def test_elementwise_validation_matches_reference(lib, ref, symbol, args):
    results = []
    for library in (lib, ref):
        err = ctypes.create_string_buffer(256)
        err.value = b"stale"
        status = getattr(library, symbol)(*args, err, len(err))
        results.append((status, err.value.decode()))
    assert results[0] == results[1]


def _raw(n, seed):
    rng = np.random.default_rng(seed)
    return [rng.normal(0, 1.5, (n, 1)).astype(np.float32), rng.normal(-4, 0.5, (n, 2)).astype(np.float32),
            rng.normal(0, 1, (n, 4)).astype(np.float32), rng.normal(-1, 1, (n, 1)).astype(np.float32),
            rng.normal(0, 1, (n, 1)).astype(np.float32)]


def test_prepare_host_bit_exact_against_reference_build():
    if not REF_PREPARE.exists():
        pytest.skip("reference host build absent")
    ref = ctypes.CDLL(str(REF_PREPARE))
    restype, argtypes = nr.SIGNATURES["hs_flashgs_prepare_npz_host_f32_v1"]
    ref.hs_flashgs_prepare_npz_host_f32_v1.restype = restype
    ref.hs_flashgs_prepare_npz_host_f32_v1.argtypes = argtypes
    raw = _raw(50_000, 3)
    raw[2][:5] = 0.0  # zero quaternion: inf/nan propagate identically
    raw[0][5:8] = np.array([[80.0], [-90.0], [np.inf]], np.float32)
    mine = ops.flashgs_prepare_host(*raw)
    theirs = ops.flashgs_prepare_host(*raw, library=ref)
    for key in mine:
        assert np.array_equal(mine[key].view(np.uint32), theirs[key].view(np.uint32)), key


def test_prepare_host_matches_golden(golden):
    data = golden("prepare_host")
    mine = ops.flashgs_prepare_host(data["in_opacity"], data["in_scaling"], data["in_rotation"],
                                    data["in_specular"], data["in_roughness"])
    for key, value in mine.items():
        assert np.array_equal(value.view(np.uint32), data[f"out_{key}"].view(np.uint32)), key


def test_prepare_host_empty_and_null(lib):
    err = ctypes.create_string_buffer(128)
    assert lib.hs_flashgs_prepare_npz_host_f32_v1(0, *([None] * 11), err, len(err)) == 0
    assert lib.hs_flashgs_prepare_npz_host_f32_v1(3, *([None] * 11), err, len(err)) == 1
    assert err.value == b"FlashGS NPZ preparation received a null host buffer"


@pytest.mark.parametrize("symbol,args,expected", [
    ("hs_b200_precise_sh_colors5_f32_v1", (None, 16, 3, None, None, None, None, 0, None), 0),
    ("hs_b200_precise_sh_colors5_f32_v1", (None, 16, 3, None, None, None, None, 10, None), 1),
    ("hs_b200_precise_sh_colors5_f32_v1", (None, 16, 4, None, None, None, None, 10, None), 3),
    ("hs_b200_precise_sh_colors5_f32_v1", (None, 8, 3, None, None, None, None, 10, None), 3),
    ("hs_b200_precise_fuse_maps_planar_f32_v1", (None, None, None, None, None, None, 0), 0),
    ("hs_b200_precise_fuse_maps_planar_f32_v1", (None, None, None, None, None, None, 10), 1),
    ("hs_b200_standard_postprocess_f32_v1", (0, 7, *[None] * 5, 0.0, *[None] * 8), 0),
    ("hs_b200_standard_postprocess_f32_v1", (4, 3, *[None] * 5, 0.0, *[None] * 8), 1),
    ("hs_b200_standard_postprocess_f32_v1", (-1, 3, *[None] * 5, 0.0, *[None] * 8), 1),
    ("hs_b200_standard_postprocess_f32_v1", (4, 3, *[None] * 5, float("inf"), *[None] * 8), 1),
    ("hs_b200_flashgs_postprocess_f32_v1", (5, 0, *[None] * 13), 0),
    ("hs_b200_flashgs_postprocess_f32_v1", (5, 2, *[None] * 13), 1),
    ("hs_b200_pixel_rays_f32_v1", (None, 8, 8, None, None, None, None), 1),
    ("hs_b200_pixel_rays_f32_v1", (None, 0, 8, None, None, None, None), 0),
    ("hs_b200_postprocess_camera_f32_v1", (None, 8, 8, 1.0, 1.0, None, None, None, None), 1),
    ("hs_b200_postprocess_camera_f32_v1", (None, 0, 8, 1.0, 1.0, None, None, None, None), 1),
    ("hs_b200_postprocess_camera_f32_v1", (None, 8, 8, float("nan"), 1.0, None, None, None, None), 1),
    ("hs_b200_postprocess_camera_f32_v1", (None, 65536, 65536, 1.0, 1.0, None, None, None, None), 3),
])
def test_fused_glue_validation(lib, symbol, args, expected):
    """Argument checks of the fused view-glue and postprocess entry points,
    before any launch (an empty image is a successful no-op); the SH checks use
    the messages of hs_rasterizer_precise_sh_to_rgb_f32_v1."""
    err = ctypes.create_string_buffer(256)
    assert getattr(lib, symbol)(*args, err, len(err)) == expected
    if expected == 3:
        prefix = "precise_sh_to_rgb" if "sh_colors5" in symbol else "postprocess_camera"
        assert err.value.decode().startswith(prefix)


def test_prepare_host_threads_bit_identical(lib):
    """Large inputs are prepared on several host threads; every element must
    equal the single-threaded result (ranges below 64K Gaussians run on the
    calling thread)."""
    n = 300_001
    raw = _raw(n, 11)
    whole = ops.flashgs_prepare_host(*raw)
    parts = [ops.flashgs_prepare_host(*[a[i:i + 50_000] for a in raw]) for i in range(0, n, 50_000)]
    for key, value in whole.items():
        joined = np.concatenate([p[key] for p in parts])
        assert np.array_equal(value.view(np.uint32), joined.view(np.uint32)), key
