"""CUDA library vs the reference library rebuilt for Blackwell, at benchmark size.

The benchmark scene (1M base + 200k reflection Gaussians, 1292x839) is
rendered by both libraries through the same C ABI on identical device
inputs, from a generic rolled camera and an orbit camera; the 6M-scene and
4K stress distributions are compared at their own resolutions. FlashGS must be
bit-identical in every output map, preprocess field, sorted pair and tile
range. The standard backend must be bit-identical in its colour and
auxiliary maps, radii and pair count, and in every visible Gaussian's centre,
ray-splat transform and normal|opacity (against the reference preprocess run
through the harness entry ref_standard_preprocess_direct); its per-Gaussian
blend weights are float atomics in both libraries and agree to a tolerance.
(The stated acceptance bar for the standard backend is max-abs 1e-5 /
mean-abs 1e-7 per channel; bit equality implies it.) Skipped when the
reference build (oracle/_ref) is absent.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from helpers import DEBUG_FIELDS, FLASHGS_OUT, bits_equal, channel_errors, within_standard_tolerance
from hybridsplat_jittor_render_b200 import NativeRendererContext, ops, scenes

pytestmark = pytest.mark.gpu


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.fixture(scope="module")
def scene():
    return scenes.make_scene("flashgs_1m")


@pytest.fixture(scope="module")
def contexts(ref_library):
    mine, ref = NativeRendererContext(0), NativeRendererContext(0, library=ref_library)
    yield mine, ref
    mine.close()
    ref.close()


def flashgs_inputs(group):
    n = group["xyz"].shape[0]
    prep = ops.flashgs_prepare_host(group["opacity"], group["scaling"], group["rotation"], group["specular"],
                                    group["roughness"])
    return [dev(group["xyz"]), dev(scenes.sh_features(group).reshape(n, 48)),
            dev(scenes.sigmoid(group["features_dc"][:, 0, :])), dev(prep["opacity"]), dev(prep["covariance"]),
            dev(prep["scaling"]), dev(prep["rotation"]), dev(prep["specular"]), dev(prep["roughness"])]


CAMERAS = {"generic": lambda: scenes.generic_camera("flashgs_1m", 3), "orbit7": lambda: scenes.orbit_camera("flashgs_1m", 7)}


@pytest.mark.parametrize("camera", sorted(CAMERAS))
@pytest.mark.parametrize("group", ["base", "reflection"])
def test_flashgs_full_size_bit_exact(scene, contexts, camera, group):
    cam = CAMERAS[camera]()
    inputs = flashgs_inputs(scene[group])
    outs, snaps = [], []
    for ctx in contexts:
        o = ops.flashgs_forward(*inputs, width=cam.width, height=cam.height, use_sh=group == "base",
                                camera_position=cam.flashgs_position, camera_rotation=cam.flashgs_rotation9,
                                focal_x=cam.fx, focal_y=cam.fy, initial_pair_capacity=2_000_000, context=ctx)
        torch.cuda.synchronize()
        outs.append([t.cpu().numpy() for t in o])
        snaps.append(ctx.flashgs_debug_snapshot())
    for i, name in enumerate((*FLASHGS_OUT, "rendered")):
        assert bits_equal(outs[0][i], outs[1][i]), name
    for name in DEBUG_FIELDS:
        assert bits_equal(snaps[0][name], snaps[1][name]), name


def test_flashgs_orbit_20_views_bit_exact(scene, contexts):
    """The FlashGS 20-view orbit of the benchmark configuration (azimuth step
    18 degrees, elevation 15, radius 4, 1292x839), both branches: every output
    map, `rendered`, preprocess record, sorted (tile | depth, index) pair and
    tile range equals the reference build's (render.cu:358-732 contract)."""
    inputs = {g: flashgs_inputs(scene[g]) for g in ("base", "reflection")}
    for view in range(20):
        cam = scenes.orbit_camera("flashgs_1m", view)
        for group in ("base", "reflection"):
            outs, snaps = [], []
            for ctx in contexts:
                o = ops.flashgs_forward(*inputs[group], width=cam.width, height=cam.height,
                                        use_sh=group == "base", camera_position=cam.flashgs_position,
                                        camera_rotation=cam.flashgs_rotation9, focal_x=cam.fx, focal_y=cam.fy,
                                        initial_pair_capacity=2_000_000, context=ctx)
                torch.cuda.synchronize()
                outs.append([t.cpu().numpy() for t in o])
                snaps.append(ctx.flashgs_debug_snapshot())
            for i, name in enumerate((*FLASHGS_OUT, "rendered")):
                assert bits_equal(outs[0][i], outs[1][i]), (view, group, name)
            for name in DEBUG_FIELDS:
                assert bits_equal(snaps[0][name], snaps[1][name]), (view, group, name)


def assert_weights_within_quantisation_bound(mine, ref, radii, label=""):
    """Per-Gaussian blend weights of the two libraries. Both are order-dependent
    float sums: the reference adds each pixel's w with a float atomicAdd
    (forward.cu:420), each add rounding by at most 2^-24 of the running sum;
    this library rounds each lane's w (two pixels) to 2^-24 fixed point (error
    <= 2^-25), sums a warp exactly in integers, then adds one float per warp.
    With M pixel contributions to a Gaussian of total weight W, each library is
    within M * 2^-24 * W + M * 2^-25 of the exact sum, so the two differ by at
    most 2^-23 * M * (W + 1). M is bounded by the pixels of the Gaussian's tile
    rectangle, (2 radius + 32)^2."""
    mine, ref = mine.reshape(-1).astype(np.float64), ref.reshape(-1).astype(np.float64)
    m = (2.0 * radii.astype(np.float64) + 32.0) ** 2
    bound = 2.0 ** -23 * m * (np.abs(ref) + 1.0)
    diff = np.abs(mine - ref)
    live = radii > 0
    worst = float(diff.max()) if diff.size else 0.0
    print(f"weights{label}: max |diff| {worst:.3g}, max |diff| / bound "
          f"{float((diff[live] / bound[live]).max()) if live.any() else 0.0:.3g}, "
          f"max relative {float((diff[live] / np.maximum(np.abs(ref[live]), 1e-30)).max()) if live.any() else 0.0:.3g}")
    assert np.all(diff[~live] == 0.0)
    assert np.all(diff <= bound), float((diff / bound).max())


def standard_inputs(group, cam):
    xyz = dev(group["xyz"])
    center = dev(scenes.standard_camera_center(cam))
    direction = ops.precise_direction(xyz, center)
    sh = dev(np.ascontiguousarray(scenes.sh_features(group).transpose(0, 2, 1)))
    colors = torch.cat([ops.precise_sh_to_rgb(sh, direction, 3), ops.precise_sigmoid(dev(group["specular"])),
                        ops.precise_sigmoid(dev(group["roughness"]))], 1).contiguous()
    return [torch.zeros(5, device="cuda"), xyz, colors, ops.precise_sigmoid(dev(group["opacity"])),
            ops.precise_exp(dev(group["scaling"])), ops.precise_normalize4(dev(group["rotation"])),
            dev(cam.world_view()), dev(cam.full_proj()), center]


STANDARD_CAMERAS = {"generic": lambda: scenes.generic_camera("standard_1m", 3),
                    "orbit7": lambda: scenes.orbit_camera("flashgs_1m", 7)}


@pytest.mark.parametrize("camera", sorted(STANDARD_CAMERAS))
@pytest.mark.parametrize("group", ["base", "reflection"])
def test_standard_full_size_bit_exact(scene, contexts, camera, group):
    cam = STANDARD_CAMERAS[camera]()
    inputs = standard_inputs(scene[group], cam)
    outs = []
    for ctx in contexts:
        o = ops.rasterize_forward(*inputs, width=cam.width, height=cam.height, scale_modifier=1.0,
                                  tan_fovx=cam.tan_fovx, tan_fovy=cam.tan_fovy, context=ctx)
        torch.cuda.synchronize()
        outs.append([t.cpu().numpy() for t in o])
    (mc, ma, mw, mr, mn), (rc, ra, rw, rr, rn) = outs
    assert bits_equal(mc, rc), channel_errors(mc, rc)
    assert bits_equal(ma, ra), channel_errors(ma, ra)
    assert within_standard_tolerance(mc, rc)
    assert np.array_equal(mr, rr) and np.array_equal(mn, rn)
    assert_weights_within_quantisation_bound(mw, rw, mr, f" {camera}/{group}")


def reference_standard_preprocess(ref_library, inputs, cam):
    """The reference preprocess kernel's per-Gaussian state for `inputs`."""
    fn = ref_library.ref_standard_preprocess_direct
    P, I, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    fn.argtypes = [I, P, P, F, P, P, P, P, P, I, I, F, F] + [P] * 7
    fn.restype = ctypes.c_int
    n = inputs[1].shape[0]
    out = {"radii": torch.zeros(n, dtype=torch.int32, device="cuda"), "points_xy": torch.zeros(n, 2, device="cuda"),
           "depths": torch.zeros(n, device="cuda"), "transmats": torch.zeros(n, 9, device="cuda"),
           "rgb": torch.zeros(n, 5, device="cuda"), "normal_opacity": torch.zeros(n, 4, device="cuda"),
           "tiles": torch.zeros(n, dtype=torch.int32, device="cuda")}
    status = fn(n, inputs[1].data_ptr(), inputs[4].data_ptr(), 1.0, inputs[5].data_ptr(), inputs[3].data_ptr(),
                inputs[2].data_ptr(), inputs[6].data_ptr(), inputs[7].data_ptr(), cam.width, cam.height,
                cam.tan_fovx, cam.tan_fovy, *[t.data_ptr() for t in out.values()])
    assert status == 0, status
    return {k: v.cpu().numpy() for k, v in out.items()}


@pytest.mark.parametrize("camera", sorted(STANDARD_CAMERAS))
@pytest.mark.parametrize("group", ["base", "reflection"])
def test_standard_preprocess_state_bit_exact(scene, contexts, ref_library, camera, group):
    cam = STANDARD_CAMERAS[camera]()
    inputs = standard_inputs(scene[group], cam)
    mine = contexts[0]
    out = ops.rasterize_forward(*inputs, width=cam.width, height=cam.height, scale_modifier=1.0,
                                tan_fovx=cam.tan_fovx, tan_fovy=cam.tan_fovy, context=mine)
    torch.cuda.synchronize()
    n = inputs[1].shape[0]
    snap = mine.standard_debug_snapshot(n)
    ref = reference_standard_preprocess(ref_library, inputs, cam)
    radii = out.radii.cpu().numpy()
    assert np.array_equal(radii, ref["radii"])
    live = radii > 0
    assert live.sum() > n // 4
    for name in ("points_xy", "transmats", "normal_opacity"):
        assert bits_equal(snap[name][live], ref[name][live]), name


def degenerate_group(seed=21):
    """A 20k-Gaussian group of the benchmark distributions with degenerate
    Gaussians mixed in: NaN and infinite positions, zero and huge scales, a
    zero quaternion, opacity 0 and 1, one at the camera centre and one just
    behind the near plane."""
    g = {k: v.copy() for k, v in scenes.make_scene("standard_1m", scale=0.02)["base"].items()}
    cam = scenes.generic_camera("standard_1m", 3)
    rng = np.random.default_rng(seed)
    idx = rng.choice(g["xyz"].shape[0], 12, replace=False)
    g["xyz"][idx[0], 1] = np.nan
    g["xyz"][idx[1], 0] = np.inf
    g["xyz"][idx[2]] = cam.center
    g["xyz"][idx[3]] = cam.center + 0.15 * cam.R[2]  # in front of the camera, inside the near plane
    g["scaling"][idx[4]] = -np.inf                   # zero scales
    g["scaling"][idx[5]] = 3.0                       # covers the screen
    g["scaling"][idx[6], 0] = 4.0
    g["rotation"][idx[7]] = 0.0
    g["opacity"][idx[8]] = -np.inf                   # opacity 0
    g["opacity"][idx[9]] = np.inf                    # opacity 1
    g["xyz"][idx[10]] = cam.center + 2.0 * cam.R[2]  # on the view axis, close
    g["scaling"][idx[10]] = 1.0
    g["specular"][idx[11]] = np.nan
    return g, cam


def same_or_both_nan(a, b):
    both = np.isnan(a) & np.isnan(b)
    return np.where(both, 0.0, a), np.where(both, 0.0, b)


def test_degenerate_gaussians_flashgs_bit_exact(contexts):
    g, cam = degenerate_group()
    with np.errstate(all="ignore"):
        inputs = flashgs_inputs(g)
    outs, snaps = [], []
    for ctx in contexts:
        o = ops.flashgs_forward(*inputs, width=cam.width, height=cam.height, use_sh=True,
                                camera_position=cam.flashgs_position, camera_rotation=cam.flashgs_rotation9,
                                focal_x=cam.fx, focal_y=cam.fy, context=ctx)
        torch.cuda.synchronize()
        outs.append([t.cpu().numpy() for t in o])
        snaps.append(ctx.flashgs_debug_snapshot())
    for i, name in enumerate((*FLASHGS_OUT, "rendered")):
        assert bits_equal(outs[0][i], outs[1][i]), name
    for name in DEBUG_FIELDS:
        assert bits_equal(snaps[0][name], snaps[1][name]), name


def test_degenerate_gaussians_standard_within_tolerance(contexts):
    g, cam = degenerate_group()
    with np.errstate(all="ignore"):
        inputs = standard_inputs(g, cam)
    outs = []
    for ctx in contexts:
        o = ops.rasterize_forward(*inputs, width=cam.width, height=cam.height, scale_modifier=1.0,
                                  tan_fovx=cam.tan_fovx, tan_fovy=cam.tan_fovy, context=ctx)
        torch.cuda.synchronize()
        outs.append([t.cpu().numpy() for t in o])
    (mc, ma, mw, mr, mn), (rc, ra, rw, rr, rn) = outs
    assert np.array_equal(mr, rr) and np.array_equal(mn, rn)
    for mine, ref in ((mc, rc), (ma, ra)):
        assert np.array_equal(np.isnan(mine), np.isnan(ref))
        a, b = same_or_both_nan(mine, ref)
        assert all(mx <= 1e-5 and mn_ <= 1e-7 for mx, mn_ in channel_errors(a, b)), channel_errors(a, b)
        assert bits_equal(mine, ref), channel_errors(a, b)
    with np.errstate(invalid="ignore"):
        finite = np.isfinite(rw.reshape(-1)) & np.isfinite(mw.reshape(-1))
    assert np.array_equal(np.isfinite(rw), np.isfinite(mw))
    assert_weights_within_quantisation_bound(mw.reshape(-1)[finite], rw.reshape(-1)[finite], mr[finite],
                                             " degenerate")


LARGE_FRAMES = {"large_6m": (0.2, 5), "stress_4k": (0.3, 1)}


@pytest.mark.parametrize("name", sorted(LARGE_FRAMES))
def test_large_and_4k_frames_bit_exact(contexts, name):
    """The 6M-scene distribution at 1920x1080 (1.2M Gaussians) and the inflated
    4K stress distribution at 3840x2160 (0.9M Gaussians): standard colour, aux,
    radii and pair counts and FlashGS outputs equal the reference build's."""
    scale, view = LARGE_FRAMES[name]
    group = scenes.make_scene(name, scale=scale)["base"]
    cam = scenes.generic_camera(name, view)
    inputs = standard_inputs(group, cam)
    outs = []
    for ctx in contexts:
        o = ops.rasterize_forward(*inputs, width=cam.width, height=cam.height, scale_modifier=1.0,
                                  tan_fovx=cam.tan_fovx, tan_fovy=cam.tan_fovy, context=ctx)
        torch.cuda.synchronize()
        outs.append([t.cpu().numpy() for t in o])
    (mc, ma, _, mr, mn), (rc, ra, _, rr, rn) = outs
    assert bits_equal(mc, rc) and bits_equal(ma, ra), (channel_errors(mc, rc), channel_errors(ma, ra))
    assert np.array_equal(mr, rr) and np.array_equal(mn, rn)
    fg = flashgs_inputs(group)
    fouts = []
    for ctx in contexts:
        o = ops.flashgs_forward(*fg, width=cam.width, height=cam.height, use_sh=True,
                                camera_position=cam.flashgs_position, camera_rotation=cam.flashgs_rotation9,
                                focal_x=cam.fx, focal_y=cam.fy, context=ctx)
        torch.cuda.synchronize()
        fouts.append([t.cpu().numpy() for t in o])
    for i, label in enumerate((*FLASHGS_OUT, "rendered")):
        assert bits_equal(fouts[0][i], fouts[1][i]), label
