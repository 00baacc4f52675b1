"""Host side of the concurrent raster entry points (hs_b200_*_forward_many_v2)
and of the one-view entry point (hs_b200_standard_view_v2).

The call structs of include/hybridsplat_b200_ext.h must match their ctypes
mirrors field by field (names, types, and the offsets a C compiler gives
them), and every call is checked, with the messages of the single-call entry
points, before any handle is used.
"""

from __future__ import annotations

import ctypes
import re
import shutil
import subprocess

import pytest

from conftest import REPO
from hybridsplat_jittor_render_b200 import native_runtime as nr
from hybridsplat_jittor_render_b200 import ops

EXT_HEADER = REPO / "include" / "hybridsplat_b200_ext.h"
C_TYPES = {
    "HsRasterizerHandle": ctypes.c_void_p, "uint64_t": ctypes.c_uint64, "int32_t": ctypes.c_int32,
    "uint32_t": ctypes.c_uint32, "float": ctypes.c_float, "double": ctypes.c_double,
    "HsB200StandardGroupV2": nr.StandardGroupV2, "HsB200FlashgsCallV2": nr.FlashgsCallV2,
}
MIRRORS = [("HsB200FlashgsCallV2", nr.FlashgsCallV2), ("HsB200RasterizerCallV2", nr.RasterizerCallV2),
           ("HsB200StandardGroupV2", nr.StandardGroupV2), ("HsB200StandardViewV2", nr.StandardViewV2),
           ("HsB200FlashgsViewV2", nr.FlashgsViewV2)]


def header_struct(name: str) -> list[tuple[str, object]]:
    body = re.search(r"typedef struct %s \{(.*?)\} %s;" % (name, name), EXT_HEADER.read_text(), re.S).group(1)
    body = re.sub(r"/\*.*?\*/", "", body, flags=re.S)
    fields = []
    for decl in filter(None, (d.strip() for d in body.split(";"))):
        ctype, field = decl.rsplit(None, 1)
        if field.startswith("*") or ctype.endswith("*"):
            fields.append((field.lstrip("*"), ctypes.c_void_p))
        else:
            fields.append((field, C_TYPES[ctype.replace("const ", "")]))
    return fields


@pytest.mark.parametrize("name,mirror", MIRRORS)
def test_call_structs_match_header(name, mirror):
    assert [(f, t) for f, t in mirror._fields_] == header_struct(name)


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs a C compiler")
def test_call_struct_offsets_match_the_c_compiler(tmp_path):
    lines = ["#include <stddef.h>", "#include <stdio.h>", '#include "hybridsplat_b200_ext.h"', "int main(void) {"]
    expected = []
    for name, mirror in MIRRORS:
        lines.append(f'printf("%zu\\n", sizeof({name}));')
        expected.append(ctypes.sizeof(mirror))
        for field, _ in mirror._fields_:
            lines.append(f'printf("%zu\\n", offsetof({name}, {field}));')
            expected.append(getattr(mirror, field).offset)
    lines += ["return 0;", "}"]
    source, binary = tmp_path / "layout.c", tmp_path / "layout"
    source.write_text("\n".join(lines))
    subprocess.run(["gcc", "-std=c99", "-I", str(REPO / "include"), str(source), "-o", str(binary)], check=True)
    printed = [int(v) for v in subprocess.run([str(binary)], check=True, capture_output=True,
                                              text=True).stdout.split()]
    assert printed == expected


def test_struct_fields_cover_the_single_call_arguments():
    flashgs = {f for f, _ in nr.FlashgsCallV2._fields_}
    raster = {f for f, _ in nr.RasterizerCallV2._fields_}
    assert flashgs == set(ops._FLASHGS_ORDER) | {"handle", "tile_row_begin", "tile_row_end"}
    assert raster == set(ops._RASTERIZER_ORDER) | {"handle", "tile_row_begin", "tile_row_end"}


@pytest.fixture(scope="module")
def lib():
    return nr.load_native_library()


def _flashgs_struct(**over):
    position, rotation, bg = (ctypes.c_float * 3)(), (ctypes.c_float * 9)(1, 0, 0, 0, 1, 0, 0, 0, 1), \
        (ctypes.c_float * 3)()
    dummy = 16
    s = nr.FlashgsCallV2(handle=dummy, point_count=0, width=64, height=48, use_sh=1, scale_modifier=1.0,
                         camera_position3=ctypes.addressof(position), camera_rotation9=ctypes.addressof(rotation),
                         focal_x=50.0, focal_y=50.0, z_far=100.0, z_near=0.01, background3=ctypes.addressof(bg),
                         initial_pair_capacity=1024, output_color3=dummy, output_other2=dummy, output_depth1=dummy,
                         output_alpha1=dummy, output_normal3=dummy, output_median_depth1=dummy,
                         output_distortion1=dummy, output_num_rendered=dummy, tile_row_begin=0,
                         tile_row_end=0xFFFFFFFF)
    for k, v in over.items():
        setattr(s, k, v)
    return s, (position, rotation, bg)


def _raster_struct(**over):
    dummy = 16
    s = nr.RasterizerCallV2(handle=dummy, point_count=0, background5=dummy, width=64, height=48,
                            scale_modifier=1.0, tan_fovx=0.5, tan_fovy=0.5, output_color5=dummy,
                            output_aux7=dummy, output_rendered=dummy, tile_row_begin=0, tile_row_end=0xFFFFFFFF)
    for k, v in over.items():
        setattr(s, k, v)
    return s


def _many(lib, symbol, structs, count=None):
    array = (type(structs[0]) * len(structs))(*structs) if structs else None
    err = ctypes.create_string_buffer(512)
    status = getattr(lib, symbol)(array, len(structs) if count is None else count, None, err, len(err))
    return status, err.value.decode()


def test_empty_and_null_batches(lib):
    for symbol in ("hs_b200_flashgs_forward_many_v2", "hs_b200_rasterizer_forward_many_v2"):
        assert _many(lib, symbol, []) == (0, "")
        assert _many(lib, symbol, [], count=2) == (1, "calls is null")


@pytest.mark.parametrize("over,expected", [
    (dict(handle=None), (1, "FlashGS received a null required handle or buffer")),
    (dict(width=0), (3, "FlashGS dimensions or scalar arguments are invalid")),
    (dict(tile_row_begin=2, tile_row_end=2), (3, "tile rows must satisfy 0 <= begin < end <= tile rows")),
    (dict(tile_row_end=4), (3, "tile rows must satisfy 0 <= begin < end <= tile rows")),
    (dict(point_count=5), (1, "non-empty FlashGS input contains a null buffer")),
])
def test_flashgs_batch_checks_every_call_first(lib, over, expected):
    good, keep_a = _flashgs_struct()
    bad, keep_b = _flashgs_struct(**over)
    # the bad call is second: the first (fake) handle must not be touched
    assert _many(lib, "hs_b200_flashgs_forward_many_v2", [good, bad]) == expected


@pytest.mark.parametrize("over,expected", [
    (dict(handle=None), (1, "rasterizer received a null required handle or buffer")),
    (dict(tan_fovx=0.0), (3, "rasterizer dimensions or scalar arguments are invalid")),
    (dict(prefiltered=2), (3, "rasterizer dimensions or scalar arguments are invalid")),
    (dict(tile_row_begin=1, tile_row_end=0), (3, "tile rows must satisfy 0 <= begin < end <= tile rows")),
    (dict(point_count=3), (1, "non-empty rasterizer input contains a null buffer")),
])
def test_rasterizer_batch_checks_every_call_first(lib, over, expected):
    assert _many(lib, "hs_b200_rasterizer_forward_many_v2", [_raster_struct(), _raster_struct(**over)]) == expected


def test_ops_rows_fields():
    assert ops._rows_fields(None) == {"tile_row_begin": 0, "tile_row_end": 0xFFFFFFFF}
    assert ops._rows_fields((1, 3)) == {"tile_row_begin": 1, "tile_row_end": 3}
    assert ops._rows_fields((0, 0xFFFFFFFF))["tile_row_end"] == 0xFFFFFFFE


def _view_struct(**over):
    dummy = 16
    group = dict(count=0, background5=dummy, colors5=dummy, output_color5=dummy, output_aux7=dummy,
                 output_rendered=dummy)
    v = nr.StandardViewV2(struct_size=ctypes.sizeof(nr.StandardViewV2), base_handle=16, reflection_handle=32,
                          width=64, height=48, tan_fovx=0.5, tan_fovy=0.5, base=nr.StandardGroupV2(**group),
                          reflection=nr.StandardGroupV2(**group), sh_coefficients=16, sh_degree=3,
                          fused_rgb3=dummy, diffuse_rgb3=dummy, reflection_rgb_map3=dummy)
    for k, val in over.items():
        if "." in k:
            outer, inner = k.split(".")
            setattr(getattr(v, outer), inner, val)
        else:
            setattr(v, k, val)
    return v


def _view(lib, v):
    err = ctypes.create_string_buffer(512)
    status = lib.hs_b200_standard_view_v2(None if v is None else ctypes.byref(v), err, len(err))
    return status, err.value.decode()


@pytest.mark.parametrize("over,expected", [
    (dict(struct_size=8), (1, "standard view is null or its struct_size is too small")),
    (dict(base_handle=None), (1, "rasterizer received a null required handle or buffer")),
    (dict(**{"reflection.output_aux7": None}), (1, "rasterizer received a null required handle or buffer")),
    (dict(width=0), (3, "rasterizer dimensions or scalar arguments are invalid")),
    (dict(**{"base.count": 5}), (1, "non-empty rasterizer input contains a null buffer")),
    (dict(reflection_handle=16), (1, "standard view needs two distinct handles")),
    (dict(sh_coefficients=4, sh_degree=2), (3, "standard view SH dimensions are invalid")),
    (dict(sh_coefficients=17), (3, "standard view SH dimensions are invalid")),
    (dict(fused_rgb3=None), (1, "standard view received a null required buffer")),
    (dict(trace=2), (3, "standard view trace must be 0 or 1")),
    (dict(trace=1, trace_coefficients=16, trace_degree=3, max_trace_depth=2),
     (3, "OptiX trace dimensions or scalars are invalid")),
    (dict(camera30=16, fov_x=float("nan")), (1, "standard view postprocess scalars must be finite")),
    (dict(camera30=16, width=70000, height=70000), (3, "postprocess_camera pixel count exceeds cuBLAS int range")),
    (dict(camera30=16), (1, "standard view postprocess received a null buffer")),
])
def test_view_checks_every_argument_before_the_handles(lib, over, expected):
    # both handles are fake: a check that passed would read them
    assert _view(lib, _view_struct(**over)) == expected


def test_view_null(lib):
    assert _view(lib, None) == (1, "standard view is null or its struct_size is too small")


def test_view_graph_stats_checks_its_pointers(lib):
    """hs_b200_view_graph_stats_v1 checks every pointer before reading the
    handle (a null or foreign handle is never dereferenced here)."""
    err = ctypes.create_string_buffer(256)
    counters = [ctypes.c_uint64(7) for _ in range(3)]
    refs = [ctypes.byref(c) for c in counters]
    for args in ((None, *refs), (16, None, refs[1], refs[2]), (16, refs[0], None, refs[2]), (16, refs[0], refs[1], None)):
        status = lib.hs_b200_view_graph_stats_v1(*args, err, len(err))
        assert (status, err.value.decode()) == (1, "view graph stats received a null pointer")
    assert [c.value for c in counters] == [7, 7, 7]


def _flashgs_view_struct(keep, **over):
    base, hold_b = _flashgs_struct(use_sh=1)
    refl, hold_r = _flashgs_struct(handle=32, use_sh=0)
    keep += [hold_b, hold_r]
    dummy = 16
    v = nr.FlashgsViewV2(struct_size=ctypes.sizeof(nr.FlashgsViewV2), base=base, reflection=refl,
                         camera_center3=dummy, fused_rgb3=dummy, diffuse_rgb3=dummy, reflection_rgb_map3=dummy)
    for k, val in over.items():
        if "." in k:
            outer, inner = k.split(".")
            setattr(getattr(v, outer), inner, val)
        else:
            setattr(v, k, val)
    return v


def _flashgs_view(lib, v):
    err = ctypes.create_string_buffer(512)
    status = lib.hs_b200_flashgs_view_v2(None if v is None else ctypes.byref(v), err, len(err))
    return status, err.value.decode()


@pytest.mark.parametrize("over,expected", [
    (dict(struct_size=8), (1, "FlashGS view is null or its struct_size is too small")),
    (dict(**{"base.handle": None}), (1, "FlashGS received a null required handle or buffer")),
    (dict(**{"reflection.width": 0}), (3, "FlashGS dimensions or scalar arguments are invalid")),
    (dict(**{"reflection.handle": 16}), (1, "FlashGS view needs two distinct handles")),
    (dict(**{"base.use_sh": 0}), (1, "FlashGS view takes the base call with SH, the reflection call with colours")),
    (dict(**{"reflection.width": 32}), (3, "FlashGS view calls must render the same whole frame")),
    (dict(**{"base.tile_row_end": 2}), (3, "FlashGS view calls must render the same whole frame")),
    (dict(camera_center3=None), (1, "FlashGS view received a null required buffer")),
    (dict(trace=3), (3, "FlashGS view trace must be 0 or 1")),
    (dict(trace=1, trace_coefficients=9, trace_degree=3), (3, "OptiX trace dimensions or scalars are invalid")),
    (dict(trace=1, trace_coefficients=16, trace_degree=3, **{"reflection.colors3": 16}),
     (1, "OptiX trace received a null non-empty buffer")),
    (dict(postprocess=2), (3, "FlashGS view postprocess must be 0 or 1")),
    (dict(postprocess=1), (1, "FlashGS view postprocess received a null buffer")),
])
def test_flashgs_view_checks_every_argument_before_the_handles(lib, over, expected):
    keep = []
    assert _flashgs_view(lib, _flashgs_view_struct(keep, **over)) == expected


def test_flashgs_view_null(lib):
    assert _flashgs_view(lib, None) == (1, "FlashGS view is null or its struct_size is too small")
