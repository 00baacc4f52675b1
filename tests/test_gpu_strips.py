"""Tile-strip rendering (frame sharding by rows of 16x16 tiles).

A strip call bins and renders only its tile rows, but every tile's list is
the full-frame list, so the strip's pixels must be bit-identical to a
full-frame call of the same backend; rows outside the strip stay untouched
and the strips' pair counts add up to the frame's.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import FLASHGS_OUT, camera_args, fixture_inputs
from hybridsplat_jittor_render_b200 import NativeRasterizerError, NativeRendererContext, multigpu, ops, scenes

pytestmark = pytest.mark.gpu
SENTINEL = float("nan")


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def flashgs_outputs(h, w):
    f = dict(dtype=torch.float32, device="cuda")
    shapes = ((3, h, w), (2, h, w), (1, h, w), (1, h, w), (3, h, w), (1, h, w), (1, h, w))
    return ops.FlashgsOutputs(*[torch.full(s, SENTINEL, **f) for s in shapes],
                              torch.zeros(1, dtype=torch.int32, device="cuda"))


def standard_outputs(h, w, n):
    f = dict(dtype=torch.float32, device="cuda")
    return ops.RasterizerOutputs(torch.full((5, h, w), SENTINEL, **f), torch.full((7, h, w), SENTINEL, **f),
                                 torch.zeros((n, 1), **f), torch.zeros(n, dtype=torch.int32, device="cuda"),
                                 torch.zeros(1, dtype=torch.int32, device="cuda"))


def nonempty_strips(height, strips):
    """The bands of `multigpu.tile_strips`; more strips than tile rows leaves
    some empty, and an empty band is rejected by the entry points."""
    return [b for b in multigpu.tile_strips((height + 15) // 16, strips) if b[1] > b[0]]


def check_strips(full_maps, strip_maps, bands, height):
    for name, full in full_maps.items():
        assembled = np.full_like(full, np.nan)
        for (b0, b1), maps in zip(bands, strip_maps):
            y0, y1 = 16 * b0, min(16 * b1, height)
            strip = maps[name]
            assert np.isnan(strip[:, :y0]).all() and np.isnan(strip[:, y1:]).all(), name  # untouched
            assembled[:, y0:y1] = strip[:, y0:y1]
        assert np.array_equal(assembled.view(np.uint32), full.view(np.uint32)), name


def flashgs_case(inputs, args, strips):
    h, w = args["height"], args["width"]
    tensors = [dev(v) for v in inputs.values()]
    with NativeRendererContext(0) as ctx:
        full = ops.flashgs_forward(*tensors, use_sh=True, context=ctx, **args)
        torch.cuda.synchronize()
        full_maps = {k: v.cpu().numpy() for k, v in zip(FLASHGS_OUT, full)}
        bands = nonempty_strips(h, strips)
        maps, pairs = [], 0
        for band in bands:
            out = ops.flashgs_forward(*tensors, use_sh=True, context=ctx, out=flashgs_outputs(h, w),
                                      tile_rows=band, **args)
            torch.cuda.synchronize()
            maps.append({k: v.cpu().numpy() for k, v in zip(FLASHGS_OUT, out)})
            pairs += int(out.rendered.item())
    check_strips(full_maps, maps, bands, h)
    assert pairs == int(full.rendered.item())


def standard_case(inputs, w, h, strips, fov=0.5):
    tensors = [dev(v) for v in inputs.values()]
    n = int(inputs["means3d"].shape[0])
    with NativeRendererContext(0) as ctx:
        full = ops.rasterize_forward(*tensors, width=w, height=h, scale_modifier=1.0, tan_fovx=fov, tan_fovy=fov,
                                     context=ctx)
        torch.cuda.synchronize()
        full_maps = {"color": full.color.cpu().numpy(), "auxiliary": full.auxiliary.cpu().numpy()}
        bands = nonempty_strips(h, strips)
        maps, pairs = [], 0
        for band in bands:
            out = ops.rasterize_forward(*tensors, width=w, height=h, scale_modifier=1.0, tan_fovx=fov,
                                        tan_fovy=fov, context=ctx, out=standard_outputs(h, w, n), tile_rows=band)
            torch.cuda.synchronize()
            maps.append({"color": out.color.cpu().numpy(), "auxiliary": out.auxiliary.cpu().numpy()})
            pairs += int(out.rendered.item())
            assert torch.equal(out.radii, full.radii)
    check_strips(full_maps, maps, bands, h)
    assert pairs == int(full.rendered.item())


@pytest.mark.parametrize("case", ["small", "ragged"])
@pytest.mark.parametrize("strips", [2, 3])
def test_flashgs_strips_match_full_frame(golden, case, strips):
    data = golden(case)
    flashgs_case(fixture_inputs(data, "flashgs", "base"), camera_args(data), strips)


@pytest.mark.parametrize("case", ["small", "ragged"])
@pytest.mark.parametrize("strips", [2, 3])
def test_standard_strips_match_full_frame(golden, case, strips):
    data = golden(case)
    w, h = (int(v) for v in data["camera_size"])
    standard_case(fixture_inputs(data, "standard", "base"), w, h, strips)


def test_strips_at_full_size():
    """Both backends on the 1M-Gaussian benchmark scene, four strips."""
    scene = scenes.make_scene("standard_1m")
    g = scene["base"]
    cam = scenes.generic_camera("standard_1m", 3)
    n = g["xyz"].shape[0]
    prep = ops.flashgs_prepare_host(g["opacity"], g["scaling"], g["rotation"], g["specular"], g["roughness"])
    fg_inputs = {"positions": g["xyz"], "shs": scenes.sh_features(g).reshape(n, 48),
                 "colors": np.zeros((n, 3), np.float32), "opacities": prep["opacity"],
                 "covariance": prep["covariance"], "scales": prep["scaling"], "rotations": prep["rotation"],
                 "specular": prep["specular"], "roughness": prep["roughness"]}
    args = dict(width=cam.width, height=cam.height, camera_position=cam.flashgs_position,
                camera_rotation=cam.flashgs_rotation9, focal_x=cam.fx, focal_y=cam.fy)
    flashgs_case(fg_inputs, args, 4)
    rng = np.random.default_rng(5)
    std_inputs = {"background": np.zeros(5, np.float32), "means3d": g["xyz"],
                  "colors": rng.random((n, 5)).astype(np.float32), "opacities": prep["opacity"],
                  "scales": prep["scaling"], "rotations": prep["rotation"], "viewmatrix": cam.world_view(),
                  "projmatrix": cam.full_proj(), "camera_position": scenes.standard_camera_center(cam)}
    standard_case(std_inputs, cam.width, cam.height, 4, fov=cam.tan_fovx)


def test_strip_range_is_checked(golden):
    data = golden("small")
    inputs = fixture_inputs(data, "flashgs", "base")
    args = camera_args(data)
    rows = (args["height"] + 15) // 16
    with NativeRendererContext(0) as ctx:
        for band in ((1, 1), (0, rows + 1), (3, 2)):
            with pytest.raises(NativeRasterizerError) as info:
                ops.flashgs_forward(*[dev(v) for v in inputs.values()], use_sh=True, context=ctx, tile_rows=band,
                                    **args)
            assert info.value.status == 3
