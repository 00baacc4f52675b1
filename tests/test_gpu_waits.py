"""Bounded device waits: a wait that runs out fails its own call, cleanly.

Every spin-wait of the sorts and scans behind a raster call (decoupled
look-back on a predecessor block's status word, the bulk copy of a sort tile)
gives up after about one second of device time. The test hook
hs_b200_test_stall_lookback_v1 makes one block of the next call's depth sort
never publish its status, so the waits of the blocks after it run out; no
GPU fault, trap or endless loop is involved. Checked here:

* the stalled call itself returns HS_STATUS_CUDA_ERROR naming the wait (not
  the call after it), within a few seconds;
* the next call on the same handle succeeds and is bit-identical to a call on
  a fresh handle (the status word is cleared per call, not per context);
* the same for the FlashGS backend and for the concurrent many_v2 entry.
"""

from __future__ import annotations

import time

import numpy as np
import pytest
import torch

from hybridsplat_jittor_render_b200 import NativeRasterizerError, NativeRendererContext, ops, scenes

pytestmark = pytest.mark.gpu

# 20000 Gaussians: ten 2048-item depth-sort tiles, so tile 1 has successors.
SPEC = scenes.SceneSpec("waits", scenes.GroupSpec(20000), scenes.GroupSpec(6000), 320, 240, 300.0)
STALL_TILE = 1
WAIT_LIMIT_S = 30.0  # the device bound is about 1 s per wait chain; generous for a busy host


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.fixture(scope="module")
def scene():
    return scenes.make_scene(SPEC)


def standard_call(scene, ctx, group="base"):
    g = scene[group]
    cam = scenes.generic_camera(SPEC, 0)
    center = dev(scenes.standard_camera_center(cam))
    n = g["xyz"].shape[0]
    colors = torch.cat([dev(np.random.default_rng(3).random((n, 3), dtype=np.float32)),
                        ops.precise_sigmoid(dev(g["specular"])), ops.precise_sigmoid(dev(g["roughness"]))], 1)
    return dict(background=torch.zeros(5, device="cuda"), means3d=dev(g["xyz"]), colors=colors.contiguous(),
                opacities=ops.precise_sigmoid(dev(g["opacity"])), scales=ops.precise_exp(dev(g["scaling"])),
                rotations=ops.precise_normalize4(dev(g["rotation"])), viewmatrix=dev(cam.world_view()),
                projmatrix=dev(cam.full_proj()), camera_position=center, width=cam.width, height=cam.height,
                scale_modifier=1.0, tan_fovx=cam.tan_fovx, tan_fovy=cam.tan_fovy, context=ctx)


def flashgs_call(scene, ctx, group="base"):
    g = scene[group]
    cam = scenes.generic_camera(SPEC, 0)
    n = g["xyz"].shape[0]
    pr = ops.flashgs_prepare_host(g["opacity"], g["scaling"], g["rotation"], g["specular"], g["roughness"])
    return dict(positions=dev(g["xyz"]), shs=dev(scenes.sh_features(g).reshape(n, 48)),
                colors=torch.zeros((n, 3), device="cuda"), opacities=dev(pr["opacity"]),
                covariance=dev(pr["covariance"]), scales=dev(pr["scaling"]), rotations=dev(pr["rotation"]),
                specular=dev(pr["specular"]), roughness=dev(pr["roughness"]), use_sh=True, width=cam.width,
                height=cam.height, camera_position=cam.flashgs_position, camera_rotation=cam.flashgs_rotation9,
                focal_x=cam.fx, focal_y=cam.fy, context=ctx)


def as_numpy(out):
    return [t.detach().cpu().numpy() for t in out]


def assert_same(out, expected):
    """Bit-identical outputs, except the standard per-Gaussian weight (float
    atomics in both libraries: order-dependent) which is compared closely."""
    for k, (a, b) in enumerate(zip(out, expected)):
        if isinstance(out, list) and len(out) == 5 and k == 2:
            np.testing.assert_allclose(a, b, rtol=1e-5, atol=1e-6)
        else:
            assert np.array_equal(a.view(np.uint8), b.view(np.uint8)), k


def expect_wait_failure(run):
    t0 = time.perf_counter()
    with pytest.raises(NativeRasterizerError) as info:
        run()
        torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert info.value.status == 4, str(info.value)
    assert "bounded device wait gave up" in str(info.value)
    assert elapsed < WAIT_LIMIT_S, f"the failing call took {elapsed:.1f} s"
    torch.cuda.synchronize()  # the context is still usable


@pytest.mark.parametrize("backend", ["standard", "flashgs"])
def test_stalled_sort_fails_the_same_call_and_the_next_call_is_clean(scene, backend):
    forward, make = (ops.rasterize_forward, standard_call) if backend == "standard" else \
        (ops.flashgs_forward, flashgs_call)
    with NativeRendererContext(0) as fresh:
        expected = as_numpy(forward(**make(scene, fresh)))
    with NativeRendererContext(0) as ctx:
        assert_same(as_numpy(forward(**make(scene, ctx))), expected)
        ctx.stall_next_sort(STALL_TILE)
        expect_wait_failure(lambda: forward(**make(scene, ctx)))
        # the status word is cleared per call: the next call is unaffected
        assert_same(as_numpy(forward(**make(scene, ctx))), expected)


def test_stalled_sort_in_concurrent_calls(scene):
    with NativeRendererContext(0) as fresh:
        expected = [as_numpy(ops.rasterize_forward(**standard_call(scene, fresh, g))) for g in ("base", "reflection")]
    with NativeRendererContext(0) as a, NativeRendererContext(0) as b:
        calls = [standard_call(scene, a, "base"), standard_call(scene, b, "reflection")]
        b.stall_next_sort(STALL_TILE)  # the reflection group has three sort tiles
        expect_wait_failure(lambda: ops.rasterize_forward_many(calls))
        outs = ops.rasterize_forward_many([standard_call(scene, a, "base"), standard_call(scene, b, "reflection")])
        for out, exp in zip(outs, expected):
            assert_same(as_numpy(out), exp)
