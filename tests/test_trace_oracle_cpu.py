"""Known answers of the CPU trace oracle (oracle/trace_oracle.c).

Hand-built scenes whose trace result follows in closed form from the
reference programs (vendor/optix_tracer/forward.cu:219-405): a ray through
the middle of a disk, two disks blended front to back, a stack of 40 faint
disks that needs three 16-hit trace steps, a disk closer than START_OFFSET
(skipped) and a ray that misses everything. These pin the oracle's
semantics before the GPU trace is compared with it.
"""

from __future__ import annotations

import math

import numpy as np
import pytest

from oracle import oracle

SH_C0 = 0.28209479177387814


def disk_scene(centres, scale, opacity, sh_dc):
    """Axis-aligned disks (identity rotation, normal +z) of the given
    scale; their triangles as in the reference's gaussian_disks."""
    centres = np.asarray(centres, np.float32)
    n = centres.shape[0]
    s3 = 3.0 * scale
    corners = np.array([[-s3, s3], [-s3, -s3], [s3, s3], [s3, -s3]], np.float32)
    vertices = np.zeros((n, 4, 3), np.float32)
    vertices[:, :, 0] = centres[:, None, 0] + corners[None, :, 0]
    vertices[:, :, 1] = centres[:, None, 1] + corners[None, :, 1]
    vertices[:, :, 2] = centres[:, None, 2]
    idx = np.arange(4 * n, dtype=np.int32).reshape(n, 4)
    triangles = np.stack([idx[:, :3], idx[:, 1:]], 1).reshape(-1, 3)
    shs = np.zeros((n, 16, 3), np.float32)
    shs[:, 0, :] = np.asarray(sh_dc, np.float32)
    inputs = {"background": np.array([0.1, 0.2, 0.3], np.float32), "means3d": centres, "shs": shs,
              "others": np.zeros((n, 2), np.float32), "opacities": np.full((n, 1), opacity, np.float32),
              "scales": np.full((n, 2), scale, np.float32),
              "rotations": np.tile(np.array([1, 0, 0, 0], np.float32), (n, 1)),
              "projmatrix": np.eye(4, dtype=np.float32), "camera_position": np.array([0, 0, -5], np.float32)}
    return inputs, vertices.reshape(-1, 3), triangles


def run(inputs, vertices, triangles, origins, directions, **kw):
    n = inputs["means3d"].shape[0]
    rays = np.asarray(origins, np.float32).reshape(-1, 3)
    assert rays.shape[0] == n  # one ray per Gaussian of the traced group
    data = dict(inputs, ray_origins=rays, ray_directions=np.asarray(directions, np.float32).reshape(-1, 3))
    return oracle.trace(data, vertices=vertices, triangles=triangles, degree=0, **kw)


def expected_color(weights, depths, colour, bg):
    t = 1.0
    c = np.zeros(3)
    d = 0.0
    for w_alpha, z in zip(weights, depths):
        w = w_alpha * t
        c += w * colour
        d += w * z
        t *= 1.0 - w_alpha
    return c + t * np.asarray(bg, np.float64), d, 1.0 - t


def test_single_disk_head_on():
    inputs, v, t = disk_scene([[0.0, 0.0, 2.0]], 0.1, 0.8, [1.0, 2.0, 3.0])
    out = run(inputs, v, t, [[0.05, 0.02, 0.0]], [[0.0, 0.0, 1.0]])
    rho = (0.05 / 0.1) ** 2 + (0.02 / 0.1) ** 2
    alpha = 0.8 * math.exp(-0.5 * rho)
    colour = np.maximum(SH_C0 * np.array([1.0, 2.0, 3.0]) + 0.5, 0.0)
    rgb, depth, acc = expected_color([alpha], [2.0], colour, inputs["background"])
    np.testing.assert_allclose(out["rgb"][0], rgb, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(out["depth"][0, 0], depth, rtol=1e-5)
    np.testing.assert_allclose(out["acc"][0, 0], acc, rtol=1e-5)
    # the normal faces the camera: -z (campos is behind the disk's +z normal)
    np.testing.assert_allclose(out["normal"][0], [0.0, 0.0, -alpha], rtol=1e-5, atol=1e-7)
    np.testing.assert_allclose(out["mid"][0, 6], depth, rtol=1e-5)  # mid: D of trace 0
    assert np.all(out["mid"][0, 16:] == 0.0)


def test_two_disks_blend_front_to_back():
    inputs, v, t = disk_scene([[0.0, 0.0, 2.0], [0.0, 0.0, 3.0]], 0.1, 0.6, [0.5, 0.5, 0.5])
    out = run(inputs, v, t, [[0.01, 0.01, 0.0], [5.0, 5.0, 0.0]], [[0.0, 0.0, 1.0], [0.0, 0.0, 1.0]])
    rho = 2 * (0.01 / 0.1) ** 2
    alpha = 0.6 * math.exp(-0.5 * rho)
    colour = np.maximum(SH_C0 * 0.5 + 0.5, 0.0) * np.ones(3)
    rgb, depth, acc = expected_color([alpha, alpha], [2.0, 3.0], colour, inputs["background"])
    np.testing.assert_allclose(out["rgb"][0], rgb, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(out["depth"][0, 0], depth, rtol=1e-5)
    np.testing.assert_allclose(out["acc"][0, 0], acc, rtol=1e-5)
    # the second ray misses both disks: background only
    np.testing.assert_allclose(out["rgb"][1], inputs["background"], rtol=0, atol=0)
    assert out["acc"][1, 0] == 0.0 and out["depth"][1, 0] == 0.0


def test_forty_faint_disks_need_three_trace_steps():
    n = 40
    centres = [[0.0, 0.0, 1.0 + k] for k in range(n)]
    inputs, v, t = disk_scene(centres, 0.2, 0.05, [0.2, 0.4, 0.6])
    origins = np.zeros((n, 3), np.float32)
    origins[1:, 0] = 100.0  # only ray 0 crosses the stack
    dirs = np.tile(np.array([0.0, 0.0, 1.0], np.float32), (n, 1))
    out = run(inputs, v, t, origins, dirs)
    alpha = 0.05 * math.exp(0.0)
    colour = np.maximum(SH_C0 * np.array([0.2, 0.4, 0.6]) + 0.5, 0.0)
    rgb, depth, acc = expected_color([alpha] * n, [1.0 + k for k in range(n)], colour, inputs["background"])
    # 40 hits: steps of 16, 16 and 8; the restart offset (1e-5) shifts no hit
    np.testing.assert_allclose(out["rgb"][0], rgb, rtol=2e-5, atol=1e-6)
    np.testing.assert_allclose(out["depth"][0, 0], depth, rtol=2e-5)
    np.testing.assert_allclose(out["acc"][0, 0], acc, rtol=2e-5)


def test_disk_closer_than_start_offset_is_skipped():
    inputs, v, t = disk_scene([[0.0, 0.0, 0.03], [0.0, 0.0, 1.0]], 0.1, 0.7, [1.0, 1.0, 1.0])
    out = run(inputs, v, t, [[0.0, 0.0, 0.0], [9.0, 9.0, 0.0]], [[0.0, 0.0, 1.0], [0.0, 0.0, 1.0]])
    colour = np.maximum(SH_C0 + 0.5, 0.0) * np.ones(3)
    rgb, depth, acc = expected_color([0.7], [1.0], colour, inputs["background"])  # only the far disk
    np.testing.assert_allclose(out["rgb"][0], rgb, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(out["depth"][0, 0], depth, rtol=1e-5)


@pytest.mark.parametrize("opacity", [0.003, 0.999])
def test_alpha_threshold_and_saturation(opacity):
    inputs, v, t = disk_scene([[0.0, 0.0, 2.0]], 0.1, opacity, [1.0, 1.0, 1.0])
    out = run(inputs, v, t, [[0.0, 0.0, 0.0]], [[0.0, 0.0, 1.0]])
    alpha = min(0.99, opacity)
    if alpha < 1.0 / 255.0:  # no contribution
        np.testing.assert_allclose(out["rgb"][0], inputs["background"], rtol=0, atol=0)
        assert out["acc"][0, 0] == 0.0
    else:
        np.testing.assert_allclose(out["acc"][0, 0], alpha, rtol=1e-6)
