"""Concurrent raster calls (hs_b200_*_forward_many_v2).

Several independent calls in one many-call (each with its own context, run
on per-context streams) must give exactly the outputs of the same calls made
one by one through the v1 entry points; per-Gaussian weights are float
atomic sums, so they are compared to rounding.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import FLASHGS_INPUTS, STANDARD_INPUTS, camera_args, fixture_inputs
from hybridsplat_jittor_render_b200 import NativeRasterizerError, NativeRendererContext, ops, scenes

pytestmark = pytest.mark.gpu


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def flashgs_item(data, group, context, **extra):
    inputs = {k: dev(v) for k, v in fixture_inputs(data, "flashgs", group).items()}
    return dict(inputs, use_sh=group == "base", context=context, **camera_args(data), **extra)


def standard_item(data, group, context, **extra):
    inputs = {k: dev(v) for k, v in fixture_inputs(data, "standard", group).items()}
    w, h = (int(v) for v in data["camera_size"])
    tan = data["camera_tan_fov"]
    return dict(inputs, width=w, height=h, scale_modifier=1.0, tan_fovx=float(tan[0]), tan_fovy=float(tan[1]),
                context=context, **extra)


def zero_outputs(h, w):
    f = dict(dtype=torch.float32, device="cuda")
    shapes = ((3, h, w), (2, h, w), (1, h, w), (1, h, w), (3, h, w), (1, h, w), (1, h, w))
    return ops.FlashgsOutputs(*[torch.zeros(s, **f) for s in shapes], torch.zeros(1, dtype=torch.int32, device="cuda"))


def same(a, b, weight_index=None):
    for i, (x, y) in enumerate(zip(a, b)):
        x, y = x.cpu().numpy(), y.cpu().numpy()
        if i == weight_index:
            np.testing.assert_allclose(x, y, rtol=1e-5, atol=1e-7)
        elif x.dtype.kind == "f":
            assert np.array_equal(x.view(np.uint32), y.view(np.uint32)), i
        else:
            assert np.array_equal(x, y), i


def check_flashgs(items):
    singles = [ops.flashgs_forward(**item) for item in items]
    torch.cuda.synchronize()
    many = ops.flashgs_forward_many(items)
    torch.cuda.synchronize()
    for s, m in zip(singles, many):
        same(s, m)


def check_standard(items):
    singles = [ops.rasterize_forward(**item) for item in items]
    torch.cuda.synchronize()
    many = ops.rasterize_forward_many(items)
    torch.cuda.synchronize()
    for s, m in zip(singles, many):
        same(s, m, weight_index=2)


@pytest.mark.parametrize("case", ["small", "ragged", "empty"])
def test_flashgs_base_and_reflection(golden, case):
    data = golden(case)
    with NativeRendererContext(0) as a, NativeRendererContext(0) as b:
        check_flashgs([flashgs_item(data, "base", a), flashgs_item(data, "reflection", b)])


@pytest.mark.parametrize("case", ["small", "ragged", "empty"])
def test_standard_base_and_reflection(golden, case):
    data = golden(case)
    with NativeRendererContext(0) as a, NativeRendererContext(0) as b:
        check_standard([standard_item(data, "base", a), standard_item(data, "reflection", b)])


def test_three_calls_with_strips_and_a_side_stream(golden):
    data = golden("small")
    rows = (int(data["camera_size"][1]) + 15) // 16
    with NativeRendererContext(0) as a, NativeRendererContext(0) as b, NativeRendererContext(0) as c:
        h, w = int(data["camera_size"][1]), int(data["camera_size"][0])

        def items():
            # strip calls leave the other rows untouched: start from zeros
            return [flashgs_item(data, "base", a, out=zero_outputs(h, w)),
                    flashgs_item(data, "reflection", b, tile_rows=(1, rows), out=zero_outputs(h, w)),
                    flashgs_item(data, "base", c, tile_rows=(0, 1), out=zero_outputs(h, w))]

        singles = [ops.flashgs_forward(**item) for item in items()]
        torch.cuda.synchronize()
        side = torch.cuda.Stream()
        many_items = items()
        torch.cuda.synchronize()
        with torch.cuda.stream(side):
            many = ops.flashgs_forward_many(many_items, stream=side.cuda_stream)
        side.synchronize()
        for s, m in zip(singles, many):
            same(s, m)


def test_full_size_scene_both_backends():
    scene = scenes.make_scene("standard_1m")
    cam = scenes.generic_camera("standard_1m", 4)
    groups = {}
    for name in ("base", "reflection"):
        g = scene[name]
        n = g["xyz"].shape[0]
        prep = ops.flashgs_prepare_host(g["opacity"], g["scaling"], g["rotation"], g["specular"], g["roughness"])
        groups[name] = (g, n, prep)
    fg_common = dict(width=cam.width, height=cam.height, camera_position=cam.flashgs_position,
                     camera_rotation=cam.flashgs_rotation9, focal_x=cam.fx, focal_y=cam.fy)
    rng = np.random.default_rng(9)
    with NativeRendererContext(0) as a, NativeRendererContext(0) as b:
        items = []
        for (name, (g, n, prep)), ctx in zip(groups.items(), (a, b)):
            inputs = dict(positions=g["xyz"], shs=scenes.sh_features(g).reshape(n, 48),
                          colors=rng.random((n, 3)).astype(np.float32), opacities=prep["opacity"],
                          covariance=prep["covariance"], scales=prep["scaling"], rotations=prep["rotation"],
                          specular=prep["specular"], roughness=prep["roughness"])
            items.append(dict({k: dev(v) for k, v in inputs.items()}, use_sh=name == "base", context=ctx,
                              **fg_common))
        check_flashgs(items)
        items = []
        for (name, (g, n, prep)), ctx in zip(groups.items(), (a, b)):
            inputs = dict(background=np.zeros(5, np.float32), means3d=g["xyz"],
                          colors=rng.random((n, 5)).astype(np.float32), opacities=prep["opacity"],
                          scales=prep["scaling"], rotations=prep["rotation"], viewmatrix=cam.world_view(),
                          projmatrix=cam.full_proj(), camera_position=scenes.standard_camera_center(cam))
            items.append(dict({k: dev(v) for k, v in inputs.items()}, width=cam.width, height=cam.height,
                              scale_modifier=1.0, tan_fovx=cam.tan_fovx, tan_fovy=cam.tan_fovy, context=ctx))
        check_standard(items)


def test_one_handle_twice_is_rejected(golden):
    data = golden("small")
    with NativeRendererContext(0) as a:
        with pytest.raises(NativeRasterizerError) as info:
            ops.flashgs_forward_many([flashgs_item(data, "base", a), flashgs_item(data, "reflection", a)])
        assert info.value.status == 1 and "its own handle" in str(info.value)
