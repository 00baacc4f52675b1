"""Graph replays of the one-view entry (hs_b200_standard_view_v2).

A view whose argument block and buffers repeat those of one of the last calls
on the same base context is captured once as a CUDA graph and then replayed
as one launch: the raster calls are sized for a pair capacity above their
recent pair counts, read the count from device memory, and the host reads
their status after the replay. Every replayed output must equal the direct
call's bit for bit (the per-Gaussian weights, float atomic sums, to rounding):
for the same view, for a new camera written into the same buffers, and after
the Gaussians grow in place so that the pair count outgrows the capture (the
replay is then rendered again directly). The direct calls themselves are
checked against the step-by-step entry points in test_gpu_view.py.
"""

from __future__ import annotations

import contextlib
import math
import os

import numpy as np
import pytest
import torch

from hybridsplat_jittor_render_b200 import NativeRendererContext, ops, scenes
from test_gpu_view import SMALL, make_view

pytestmark = pytest.mark.gpu

MEDIUM = scenes.SceneSpec("view_graph_medium", scenes.GroupSpec(20000), scenes.GroupSpec(4000), 320, 240, 150.0)


@contextlib.contextmanager
def graphs(enabled: bool):
    old = os.environ.get("HS_B200_VIEW_GRAPHS")
    os.environ["HS_B200_VIEW_GRAPHS"] = "1" if enabled else "0"
    try:
        yield
    finally:
        if old is None:
            del os.environ["HS_B200_VIEW_GRAPHS"]
        else:
            os.environ["HS_B200_VIEW_GRAPHS"] = old


def call(base, refl, camera, cam, ctx, ctx_r, stream, *, post, out=None):
    fov_x, fov_y = 2.0 * math.atan(cam.tan_fovx), 2.0 * math.atan(cam.tan_fovy)
    with torch.cuda.stream(stream):
        return ops.standard_view(base, refl, camera["viewmatrix"], camera["projmatrix"], camera["camera_position"],
                                 camera["background"], width=cam.width, height=cam.height, tan_fovx=cam.tan_fovx,
                                 tan_fovy=cam.tan_fovy, sh_degree=3, base_context=ctx, reflection_context=ctx_r,
                                 postprocess={"fov_x": fov_x, "fov_y": fov_y, "depth_ratio": 0.0} if post else None,
                                 stream=stream.cuda_stream, out=out)


def snapshot(one, stream) -> dict[str, np.ndarray]:
    stream.synchronize()
    got = {}
    for name in ("base", "reflection"):
        for field in ("color", "auxiliary", "weight", "radii", "rendered"):
            got[f"{name}.{field}"] = getattr(getattr(one, name), field)
    for field in ("base_colors", "reflection_colors", "reflection_rotation", "reflection_normal", "reflection_rays"):
        got[field] = getattr(one, field)
    for group in ("fused", "camera", "maps"):
        for k, t in (getattr(one, group) or {}).items():
            got[f"{group}.{k}"] = t
    return {k: t.detach().cpu().numpy().copy() for k, t in got.items()}


def same(got, want):
    assert got.keys() == want.keys()
    for k in want:
        a, b = got[k], want[k]
        assert a.shape == b.shape, k
        if k.endswith(".weight"):
            np.testing.assert_allclose(a, b, rtol=1e-5, atol=1e-7, err_msg=k)
        elif a.dtype.kind == "f":
            assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), k
        else:
            assert np.array_equal(a, b), k


def direct(base, refl, camera, cam, stream, *, post):
    """The view through the direct path, on contexts of its own."""
    with graphs(False), NativeRendererContext(0) as ctx, NativeRendererContext(0) as ctx_r:
        result = snapshot(call(base, refl, camera, cam, ctx, ctx_r, stream, post=post), stream)
        assert ops.view_graph_stats(ctx) == {"captures": 0, "replays": 0, "reruns": 0}
        return result


def stats_after(ctx, before, **delta):
    """The context's replay counters, checked against `before` plus `delta`
    (counters not named must not move)."""
    now = ops.view_graph_stats(ctx)
    assert now == {k: before[k] + delta.get(k, 0) for k in before}, (before, now)
    return now


# The first calls on fresh contexts size their buffers, which changes the key
# (it holds the buffers' addresses): a view is captured at the latest on its
# third call with unchanged buffers, and every later call replays.
WARM_CALLS = 3


@pytest.mark.parametrize("post", [True, False])
def test_replays_equal_the_direct_call(post):
    cam = scenes.generic_camera(SMALL, 1)
    base, refl, _, camera = make_view(SMALL, cam)
    stream = torch.cuda.Stream()
    want = direct(base, refl, camera, cam, stream, post=post)
    with graphs(True), NativeRendererContext(0) as ctx, NativeRendererContext(0) as ctx_r:
        first = call(base, refl, camera, cam, ctx, ctx_r, stream, post=post)
        same(snapshot(first, stream), want)
        for _ in range(WARM_CALLS):
            same(snapshot(call(base, refl, camera, cam, ctx, ctx_r, stream, post=post, out=first), stream), want)
        warm = ops.view_graph_stats(ctx)
        assert warm["captures"] == 1 and warm["replays"] >= 1 and warm["reruns"] == 0, warm
        for _ in range(3):
            same(snapshot(call(base, refl, camera, cam, ctx, ctx_r, stream, post=post, out=first), stream), want)
        stats_after(ctx, warm, replays=3)


def test_views_cycling_through_output_sets_replay():
    """Three output sets used in turn (a read-back pipeline): every set's
    argument block is captured and replayed."""
    cam = scenes.generic_camera(SMALL, 1)
    base, refl, _, camera = make_view(SMALL, cam)
    stream = torch.cuda.Stream()
    want = direct(base, refl, camera, cam, stream, post=True)
    with graphs(True), NativeRendererContext(0) as ctx, NativeRendererContext(0) as ctx_r:
        outs = [call(base, refl, camera, cam, ctx, ctx_r, stream, post=True) for _ in range(3)]
        for o in outs:
            same(snapshot(o, stream), want)
        for _ in range(WARM_CALLS):
            for o in outs:
                same(snapshot(call(base, refl, camera, cam, ctx, ctx_r, stream, post=True, out=o), stream), want)
        warm = ops.view_graph_stats(ctx)
        assert warm["captures"] == 3 and warm["reruns"] == 0, warm
        for _ in range(2):
            for o in outs:
                same(snapshot(call(base, refl, camera, cam, ctx, ctx_r, stream, post=True, out=o), stream), want)
        stats_after(ctx, warm, replays=6)


def test_replay_follows_a_camera_written_in_place():
    cams = [scenes.generic_camera(SMALL, s) for s in (1, 3, 4)]
    base, refl, _, camera = make_view(SMALL, cams[0])
    stream = torch.cuda.Stream()
    views = [make_view(SMALL, cam)[3] for cam in cams]
    with graphs(True), NativeRendererContext(0) as ctx, NativeRendererContext(0) as ctx_r:
        first = call(base, refl, camera, cams[0], ctx, ctx_r, stream, post=True)
        for _ in range(WARM_CALLS):
            call(base, refl, camera, cams[0], ctx, ctx_r, stream, post=True, out=first)
        warm = ops.view_graph_stats(ctx)
        for cam, c in zip(cams[1:], views[1:]):
            with torch.cuda.stream(stream):
                for k in ("viewmatrix", "projmatrix", "camera_position"):
                    camera[k].copy_(c[k])
            got = snapshot(call(base, refl, camera, cam, ctx, ctx_r, stream, post=True, out=first), stream)
            same(got, direct(base, refl, c, cam, stream, post=True))
        stats_after(ctx, warm, replays=2)


def test_replay_that_outgrows_its_pair_capacity_renders_again():
    cam = scenes.generic_camera(MEDIUM, 2)
    base, refl, _, camera = make_view(MEDIUM, cam)
    stream = torch.cuda.Stream()
    with graphs(True), NativeRendererContext(0) as ctx, NativeRendererContext(0) as ctx_r:
        first = call(base, refl, camera, cam, ctx, ctx_r, stream, post=True)
        for _ in range(WARM_CALLS):
            call(base, refl, camera, cam, ctx, ctx_r, stream, post=True, out=first)
        warm = ops.view_graph_stats(ctx)
        assert warm["replays"] >= 1, warm
        # the same buffers, Gaussians eight times larger: far more pairs than captured for
        with torch.cuda.stream(stream):
            base["scales"].mul_(8.0)
            refl["scales"].mul_(8.0)
        want = direct(base, refl, camera, cam, stream, post=True)
        got = snapshot(call(base, refl, camera, cam, ctx, ctx_r, stream, post=True, out=first), stream)
        same(got, want)
        grown = stats_after(ctx, warm, replays=1, reruns=1)
        # the grown buffers: direct calls, then a new capture that replays
        for _ in range(WARM_CALLS + 1):
            got = snapshot(call(base, refl, camera, cam, ctx, ctx_r, stream, post=True, out=first), stream)
            same(got, want)
        end = ops.view_graph_stats(ctx)
        assert end["reruns"] == grown["reruns"] and end["captures"] == grown["captures"] + 1, (grown, end)
        got = snapshot(call(base, refl, camera, cam, ctx, ctx_r, stream, post=True, out=first), stream)
        same(got, want)
        stats_after(ctx, end, replays=1)


def test_views_on_the_legacy_default_stream_run_directly():
    """A capture needs a stream other than the legacy default stream: the
    capture fails, the key is remembered as not replayable, and every call
    renders directly."""
    cam = scenes.generic_camera(SMALL, 1)
    base, refl, _, camera = make_view(SMALL, cam)
    fov_x, fov_y = 2.0 * math.atan(cam.tan_fovx), 2.0 * math.atan(cam.tan_fovy)
    legacy = torch.cuda.default_stream()
    want = direct(base, refl, camera, cam, torch.cuda.Stream(), post=True)
    with graphs(True), NativeRendererContext(0) as ctx, NativeRendererContext(0) as ctx_r:
        out = None
        for _ in range(WARM_CALLS + 2):
            out = ops.standard_view(base, refl, camera["viewmatrix"], camera["projmatrix"],
                                    camera["camera_position"], camera["background"], width=cam.width,
                                    height=cam.height, tan_fovx=cam.tan_fovx, tan_fovy=cam.tan_fovy, sh_degree=3,
                                    base_context=ctx, reflection_context=ctx_r,
                                    postprocess={"fov_x": fov_x, "fov_y": fov_y, "depth_ratio": 0.0}, out=out)
            same(snapshot(out, legacy), want)
        stats = ops.view_graph_stats(ctx)
        assert stats["captures"] <= 1 and stats["replays"] == 0 and stats["reruns"] == 0, stats
