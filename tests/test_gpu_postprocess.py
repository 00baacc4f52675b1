"""Fused raw-map postprocess of a view.

* The per-view camera matrices (inverse intrinsics, camera-to-world rotation
  and origin) and the world-space pixel rays equal, bit for bit, those the
  reference library's own helpers produce (its general inverse and its TF32
  N x 3 by 3 x 3 GEMM, applied as depth_to_normal applies them).
* The fused standard and FlashGS postprocess equal, bit for bit, the CPU
  restatement of the sessions' operation sequence (oracle/postprocess.py) on
  the same raster outputs and rays, for the benchmark distributions and for a
  frame with empty (alpha 0) pixels and non-finite median depths (NaN payloads
  aside: the GPU's quiet NaN differs from numpy's).

Skipped when the reference build (oracle/_ref) is absent.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from helpers import bits_equal
from hybridsplat_jittor_render_b200 import NativeRendererContext, ops, scenes
from oracle import postprocess as restated
from test_gpu_reference import flashgs_inputs, standard_inputs

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def contexts(ref_library):
    mine, ref = NativeRendererContext(0), NativeRendererContext(0, library=ref_library)
    yield mine, ref
    mine.close()
    ref.close()


def camera_inputs(cam):
    """width, height, FoVx, FoVy and world_view_transform as the session holds them."""
    return (cam.width, cam.height, 2.0 * math.atan(cam.tan_fovx), 2.0 * math.atan(cam.tan_fovy),
            torch.from_numpy(np.ascontiguousarray(cam.world_view())).cuda())


def host(t: torch.Tensor) -> np.ndarray:
    return t.cpu().numpy()


def bits_equal_any_nan(a: np.ndarray, b: np.ndarray) -> bool:
    """Bit equality with every NaN equal to every other: the GPU's quiet NaN is
    0x7fffffff, numpy's on x86 0xffc00000."""
    if not np.array_equal(np.isnan(a), np.isnan(b)):
        return False
    return bits_equal(np.where(np.isnan(a), np.float32(0), a), np.where(np.isnan(b), np.float32(0), b))


@pytest.mark.parametrize("camera", ["generic", "orbit", "stress_4k"])
def test_camera_matrices_and_rays_match_reference_helpers(contexts, camera):
    """The rays of this library's one-kernel MMA path against the reference's
    two cuBLAS TF32 GEMMs; at 3840 x 2160 pixel columns above 2048 are not
    TF32 values, so the operand rounding is exercised too."""
    mine, ref = contexts
    cam = {"generic": lambda: scenes.generic_camera("standard_1m", 3),
           "orbit": lambda: scenes.orbit_camera("standard_1m", 4),
           "stress_4k": lambda: scenes.generic_camera("stress_4k", 1)}[camera]()
    w, h, fov_x, fov_y, wv = camera_inputs(cam)
    ours = ops.postprocess_camera(w, h, fov_x, fov_y, wv, context=mine)
    theirs = ops.postprocess_camera(w, h, fov_x, fov_y, wv, context=ref)
    for name in ours:
        assert bits_equal(host(ours[name]), host(theirs[name])), name
    rays = ops.pixel_rays(w, h, ours["inverse_intrinsics"], ours["rotation"], context=mine)
    ys, xs = torch.meshgrid(torch.arange(h, dtype=torch.float32), torch.arange(w, dtype=torch.float32),
                            indexing="ij")
    pixels = torch.stack([xs, ys, torch.ones_like(xs)], -1).reshape(-1, 3).cuda()
    camera_rays = ops.precise_matmul_nt_n3k3(pixels, theirs["inverse_intrinsics"], context=ref)
    reference_rays = ops.precise_matmul_nt_n3k3(camera_rays, theirs["rotation"], context=ref)
    torch.cuda.synchronize()
    assert bits_equal(host(rays), host(reference_rays))


@pytest.mark.parametrize("camera", ["generic", "stress_4k", "tiny"])
def test_camera_entry_on_a_side_stream_matches_the_helpers(contexts, camera):
    """hs_b200_postprocess_camera_f32_v1 on a side stream: matrices and rays
    bit-identical to postprocess_camera + pixel_rays on the legacy stream,
    also for an image under 8 pixels (the cuBLAS path)."""
    mine = contexts[0]
    if camera == "tiny":
        spec = scenes.SceneSpec("tiny", scenes.GroupSpec(1), scenes.GroupSpec(1), 3, 2, 2.5)
        cam = scenes.generic_camera(spec, 2)
    else:
        cam = scenes.generic_camera("standard_1m" if camera == "generic" else camera, 3)
    w, h, fov_x, fov_y, wv = camera_inputs(cam)
    m = ops.postprocess_camera(w, h, fov_x, fov_y, wv, context=mine)
    rays = ops.pixel_rays(w, h, m["inverse_intrinsics"], m["rotation"], context=mine)
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    for _ in range(2):  # the second call reuses the entry's workspace region
        with torch.cuda.stream(side):
            got = ops.postprocess_camera_rays(w, h, fov_x, fov_y, wv, context=mine, stream=side.cuda_stream)
        side.synchronize()
        for name in ("inverse_intrinsics", "rotation", "origin", "normal_rotation"):
            assert bits_equal(host(got[name].contiguous()), host(m[name])), name
        assert bits_equal(host(got["rays"]), host(rays))


def tf32_halfway_values(rng, count):
    """Values whose low 13 mantissa bits are exactly half a TF32 ulp, with
    even and odd TF32 mantissas and both signs: rounding half away from zero
    and half to even disagree on half of them."""
    bits = rng.integers(0x30000000, 0x50000000, count, dtype=np.uint32)
    bits = (bits & np.uint32(0xffffe000)) | np.uint32(0x1000)
    bits |= rng.integers(0, 2, count, dtype=np.uint32) << np.uint32(31)
    return bits.view(np.float32)


@pytest.mark.parametrize("rows", [1, 5, 7, 8, 4096, 1_000_003])
def test_tf32_matmul_matches_reference_cublas(contexts, rows):
    """precise_matmul_nt_n3k3 (MMA kernel here from 8 rows, cublasSgemm with
    TF32 tensor-op math in the reference) bit for bit on rows of mixed
    magnitudes, TF32 halfway values (rounding half away from zero would
    disagree on them), zeros and a ragged tail."""
    mine, ref = contexts
    rng = np.random.default_rng(rows)
    left = (rng.standard_normal((rows, 3)) * np.exp2(rng.integers(-24, 24, (rows, 3)))).astype(np.float32)
    flat = left.reshape(-1)
    k = min(flat.size, 30_000)
    flat[:k] = tf32_halfway_values(rng, k)
    if rows > 4:
        left[3] = 0.0
        left[4] = [-0.0, 1.0, -1.0]
    for right in (rng.standard_normal((3, 3)).astype(np.float32),
                  tf32_halfway_values(rng, 9).reshape(3, 3)):
        a = ops.precise_matmul_nt_n3k3(torch.from_numpy(left).cuda(), torch.from_numpy(right).cuda(),
                                       context=mine)
        b = ops.precise_matmul_nt_n3k3(torch.from_numpy(left).cuda(), torch.from_numpy(right).cuda(),
                                       context=ref)
        torch.cuda.synchronize()
        assert bits_equal(host(a), host(b))


def standard_view(ctx, group, cam):
    inputs = standard_inputs(group, cam)
    out = ops.rasterize_forward(*inputs, width=cam.width, height=cam.height, scale_modifier=1.0,
                                tan_fovx=cam.tan_fovx, tan_fovy=cam.tan_fovy, context=ctx)
    w, h, fov_x, fov_y, wv = camera_inputs(cam)
    matrices = ops.postprocess_camera(w, h, fov_x, fov_y, wv, context=ctx)
    rays = ops.pixel_rays(w, h, matrices["inverse_intrinsics"], matrices["rotation"], context=ctx)
    return out, matrices, rays


@pytest.mark.parametrize("ratio", [0.0, 0.3])
def test_standard_postprocess_matches_restatement(contexts, ratio):
    ctx = contexts[0]
    scene = scenes.make_scene("standard_1m", scale=0.1)
    cam = scenes.generic_camera("standard_1m", 3)
    out, matrices, rays = standard_view(ctx, scene["base"], cam)
    # an empty block (alpha 0, depth 0 and a non-finite median) next to the rendered pixels
    aux = out.auxiliary.clone()
    aux[:, 100:180, 200:330] = 0.0
    aux[5, 100:140, 200:260] = float("nan")
    aux[5, 140:180, 200:260] = float("-inf")
    maps = ops.standard_postprocess(out.color, aux, rays, matrices["origin"], matrices["normal_rotation"],
                                    depth_ratio=ratio)
    torch.cuda.synchronize()
    expect = restated.standard_postprocess(host(out.color), host(aux), host(rays), host(matrices["origin"]),
                                           host(matrices["normal_rotation"]), ratio)
    alpha = host(aux)[1]
    assert (alpha > 0).mean() > 0.5 and (alpha == 0).any()
    assert set(maps) == set(expect)
    for name, value in expect.items():
        assert bits_equal_any_nan(host(maps[name]), value), name
    # interior surface normals are unit vectors scaled by alpha
    surf = host(maps["surf_norm_map"]).reshape(cam.height, cam.width, 3)[1:-1, 1:-1]
    a = alpha[1:-1, 1:-1]
    covered = a > 0.5
    lengths = np.linalg.norm(surf[covered].astype(np.float64), axis=-1) / a[covered]
    assert covered.sum() > 100_000 and np.mean(np.abs(lengths - 1.0) < 1e-5) > 0.999


def test_flashgs_postprocess_matches_restatement(contexts):
    ctx = contexts[0]
    group = scenes.make_scene("flashgs_1m", scale=0.1)["base"]
    cam = scenes.generic_camera("flashgs_1m", 3)
    out = ops.flashgs_forward(*flashgs_inputs(group), width=cam.width, height=cam.height, use_sh=True,
                              camera_position=cam.flashgs_position, camera_rotation=cam.flashgs_rotation9,
                              focal_x=cam.fx, focal_y=cam.fy, context=ctx)
    w, h, fov_x, fov_y, wv = camera_inputs(cam)
    matrices = ops.postprocess_camera(w, h, fov_x, fov_y, wv, context=ctx)
    maps = ops.flashgs_postprocess(out, matrices["normal_rotation"])
    torch.cuda.synchronize()
    expect = restated.flashgs_postprocess(host(out.color), host(out.other), host(out.depth), host(out.alpha),
                                          host(out.normal), host(matrices["normal_rotation"]))
    assert set(maps) == set(expect)
    for name, value in expect.items():
        assert bits_equal(host(maps[name]), value), name
