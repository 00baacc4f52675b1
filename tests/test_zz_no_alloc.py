"""The allocation-free standard forward against the context entry point.

hs_b200_rasterizer_forward_noalloc_f32_v1 runs the kernels of
hs_rasterizer_forward_f32_v1 with its scratch in a fixed device array; on the
same inputs its outputs must agree with the context path within the standard
backend's tolerance (they are expected to be identical), on two calls in a
row. Kept in its own file, collected last, so it also runs after every other
GPU test in the same process.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from helpers import STANDARD_MAX_ABS, fixture_inputs
from hybridsplat_jittor_render_b200 import NativeRendererContext, ops, scenes
from hybridsplat_jittor_render_b200 import native_runtime as nr

pytestmark = pytest.mark.gpu


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def noalloc_forward(lib, inputs, w, h, point_count=None):
    f = dict(dtype=torch.float32, device="cuda")
    n = int(inputs["means3d"].shape[0])
    color = torch.empty((5, h, w), **f)
    aux = torch.empty((7, h, w), **f)
    weight = torch.empty((n, 1), **f)
    radii = torch.empty((n,), dtype=torch.int32, device="cuda")
    rendered = torch.empty((1,), dtype=torch.int32, device="cuda")
    t = {k: dev(v) for k, v in inputs.items()}
    err = nr.error_buffer()
    status = lib.hs_b200_rasterizer_forward_noalloc_f32_v1(
        torch.cuda.current_device(), n if point_count is None else point_count,
        t["background"].data_ptr(), w, h, t["means3d"].data_ptr(), t["colors"].data_ptr(),
        t["opacities"].data_ptr(), t["scales"].data_ptr(), 1.0, t["rotations"].data_ptr(),
        t["viewmatrix"].data_ptr(), t["projmatrix"].data_ptr(), t["camera_position"].data_ptr(), 0.5,
        0.5, 0,
        color.data_ptr(), aux.data_ptr(), weight.data_ptr(), radii.data_ptr(), rendered.data_ptr(),
        err, len(err))
    torch.cuda.synchronize()
    return status, err.value.decode(), (color, aux, weight, radii, rendered)


@pytest.mark.parametrize("case", ["small", "ragged", "background"])
@pytest.mark.parametrize("group", ["base", "reflection"])
def test_noalloc_matches_context_path_twice(golden, case, group):
    data = golden(case)
    inputs = fixture_inputs(data, "standard", group)
    w, h = (int(v) for v in data["camera_size"])
    lib = nr.load_native_library()
    with NativeRendererContext(0) as ctx:
        ref = ops.rasterize_forward(*[dev(v) for v in inputs.values()], width=w, height=h,
                                    scale_modifier=1.0, tan_fovx=0.5, tan_fovy=0.5, context=ctx)
        torch.cuda.synchronize()
    for _ in range(2):
        status, message, (color, aux, weight, radii, rendered) = noalloc_forward(lib, inputs, w, h)
        assert status == 0, message
        assert int(rendered.item()) == int(ref.rendered.item())
        assert torch.equal(radii, ref.radii)
        assert torch.equal(color, ref.color) and torch.equal(aux, ref.auxiliary)
        np.testing.assert_allclose(weight.cpu().numpy(), ref.weight.cpu().numpy(), rtol=1e-5,
                                   atol=STANDARD_MAX_ABS)


def test_noalloc_rejects_sizes_beyond_its_limits(golden):
    data = golden("small")
    inputs = fixture_inputs(data, "standard", "base")
    lib = nr.load_native_library()
    status, message, _ = noalloc_forward(lib, inputs, 4096, 2048)  # 32768 tiles > 4096
    assert status == 3 and "tile count" in message and "4096" in message
    big = {k: v for k, v in inputs.items()}
    for key in ("means3d", "colors", "opacities", "scales", "rotations"):
        big[key] = np.concatenate([inputs[key]] * 9, axis=0)  # 18000 Gaussians > 16384
    status, message, _ = noalloc_forward(lib, big, 96, 72)
    assert status == 3 and "point_count" in message and "16384" in message


def large_footprint_inputs(count: int = 3000) -> tuple[dict, int, int]:
    """`count` near-opaque Gaussians of scale 0.5 around the origin, seen from
    distance 4 on a 1024x1024 view (exactly 4096 tiles): each covers hundreds
    of tiles, so the emitted pairs far exceed the fixed pair limit."""
    spec = scenes.SceneSpec("noalloc_pairs", scenes.GroupSpec(count), scenes.GroupSpec(1), 1024, 1024, 800.0)
    cam = scenes.look_at_camera(spec, (0.0, -4.0, 1.0))
    rng = np.random.default_rng(11)
    q = rng.normal(size=(count, 4)).astype(np.float32)
    q /= np.linalg.norm(q, axis=1, keepdims=True)
    inputs = {
        "background": np.zeros(5, np.float32),
        "means3d": rng.normal(0.0, 0.3, (count, 3)).astype(np.float32),
        "colors": rng.random((count, 5), dtype=np.float32),
        "opacities": np.full((count, 1), 0.99, np.float32),
        "scales": np.full((count, 2), 0.5, np.float32),
        "rotations": q,
        "viewmatrix": cam.world_view(),
        "projmatrix": cam.full_proj(),
        "camera_position": scenes.standard_camera_center(cam),
    }
    return inputs, spec.width, spec.height


def test_noalloc_rejects_too_many_emitted_pairs_then_recovers(golden):
    lib = nr.load_native_library()
    inputs, w, h = large_footprint_inputs()
    assert inputs["means3d"].shape[0] <= 16384 and ((w + 15) // 16) * ((h + 15) // 16) <= 4096
    with NativeRendererContext(0) as ctx:  # the context path has no pair limit
        ref = ops.rasterize_forward(*[dev(v) for v in inputs.values()], width=w, height=h, scale_modifier=1.0,
                                    tan_fovx=0.5, tan_fovy=0.5, context=ctx)
        torch.cuda.synchronize()
        assert int(ref.rendered.item()) > 262144
    status, message, _ = noalloc_forward(lib, inputs, w, h)
    assert status == 3 and "emitted pair count" in message and "262144" in message, message
    # Nothing was written past the scratch array: a normal call that follows
    # still equals the context path.
    data = golden("small")
    small = fixture_inputs(data, "standard", "base")
    sw, sh = (int(v) for v in data["camera_size"])
    with NativeRendererContext(0) as ctx:
        ref = ops.rasterize_forward(*[dev(v) for v in small.values()], width=sw, height=sh, scale_modifier=1.0,
                                    tan_fovx=0.5, tan_fovy=0.5, context=ctx)
        torch.cuda.synchronize()
    status, message, (color, aux, weight, radii, rendered) = noalloc_forward(lib, small, sw, sh)
    assert status == 0, message
    assert int(rendered.item()) == int(ref.rendered.item())
    assert torch.equal(radii, ref.radii)
    assert torch.equal(color, ref.color) and torch.equal(aux, ref.auxiliary)


def test_noalloc_restores_the_callers_device(golden):
    lib = nr.load_native_library()
    data = golden("small")
    inputs = fixture_inputs(data, "standard", "base")
    w, h = (int(v) for v in data["camera_size"])
    before = torch.cuda.current_device()
    status, message, _ = noalloc_forward(lib, inputs, w, h)
    assert status == 0, message
    assert torch.cuda.current_device() == before
