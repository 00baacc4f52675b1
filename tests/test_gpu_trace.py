"""The reflection trace (hs_optix_build_scene_v1 / hs_optix_trace_f32_v1) on a
B200 against the CPU trace oracle (oracle/trace_oracle.c).

The library traces on CUDA cores: its scene is a BVH over the disk triangles
of the reflective Gaussians, each trace step collects the 16 nearest hits
and shades them as the reference's OptiX programs do. The oracle restates
the same programs by brute force over every triangle with the same
arithmetic (only expf differs), so the two agree to a tolerance ray by ray;
neither is pinned against the reference's OptiX trace, which needs an OptiX
SDK this build does not have. Covered: random scenes with the benchmark
distributions and denser ones (several 16-hit steps per ray), the second
bounce with auxiliary channels, the start_from_first branch, a sample of
the full 200k-Gaussian benchmark group, and the entry points' argument,
signature-cache, release and stats behaviour.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from hybridsplat_jittor_render_b200 import NativeRasterizerError, NativeRendererContext, ops, scenes
from oracle import oracle

pytestmark = pytest.mark.gpu

# rgb of a ray agrees within this bound unless an alpha/transmittance
# threshold decision flips (expf differs by ulps between CUDA and libm)
RGB_TOL = 1e-5
AGREE_FRACTION = 0.995


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def make_case(count: int, xyz_sigma: float, log_scale, seed: int = 0, camera_seed: int = 2):
    """A reflective group with its trace inputs: rays from the library's
    reflection prefix/suffix (origin = centre + 0.05 direction), SH degree 3,
    activated opacity/scale/rotation, disks as in the reference session."""
    spec = scenes.SceneSpec("trace_case", scenes.GroupSpec(1), scenes.GroupSpec(count, xyz_sigma=xyz_sigma,
                                                                                log_scale=log_scale),
                            640, 480, 500.0, seed=seed)
    g = scenes.make_scene(spec)["reflection"]
    cam = scenes.generic_camera(spec, camera_seed)
    center = dev(scenes.standard_camera_center(cam))
    xyz, rot_raw = dev(g["xyz"]), dev(g["rotation"])
    scale = ops.precise_exp(dev(g["scaling"]))
    rot = ops.precise_reflection_prefix(rot_raw)
    packed = ops.precise_reflection_suffix(xyz, center, rot[:, :, 2].contiguous())
    inputs = {
        "ray_origins": packed[:, 12:15].contiguous(), "ray_directions": packed[:, 9:12].contiguous(),
        "background": torch.tensor([0.05, 0.1, 0.15], device="cuda"), "means3d": xyz,
        "shs": dev(scenes.sh_features(g)),
        "others": torch.cat([ops.precise_sigmoid(dev(g["specular"])), ops.precise_sigmoid(dev(g["roughness"]))], 1),
        "opacities": ops.precise_sigmoid(dev(g["opacity"])), "scales": scale,
        "rotations": ops.precise_normalize4(rot_raw), "viewmatrix": dev(cam.world_view()),
        "projmatrix": dev(cam.full_proj()), "camera_position": center,
    }
    vertices, triangles = ops.gaussian_disks(xyz, rot_raw, scale)
    return inputs, vertices, triangles


def gpu_trace(ctx, inputs, vertices, triangles, **kw):
    ops.build_trace_scene(vertices, triangles, scene_signature=7, context=ctx)
    out = ops.trace_reflection(*inputs.values(), degree=3, context=ctx, **kw)
    torch.cuda.synchronize()
    return {k: getattr(out, k).cpu().numpy() for k in ("rgb", "depth", "acc", "normal", "dist", "aux", "mid")}


def cpu_trace(inputs, vertices, triangles, ray_ids=None, **kw):
    host = {k: v.cpu().numpy() for k, v in inputs.items() if k != "viewmatrix"}
    return oracle.trace(host, vertices=vertices.cpu().numpy(), triangles=triangles.cpu().numpy(), degree=3,
                        ray_ids=ray_ids, **kw)


def compare(gpu, cpu, ids=None, min_hit_fraction=0.2):
    sel = slice(None) if ids is None else ids
    g_rgb, c_rgb = gpu["rgb"][sel], cpu["rgb"][sel]
    assert np.isfinite(g_rgb).all()
    diff = np.abs(g_rgb.astype(np.float64) - c_rgb).max(axis=1)
    agree = float(np.mean(diff <= RGB_TOL))
    hit = float(np.mean(cpu["acc"][sel, 0] > 0))
    print(f"trace: {len(diff)} rays, {hit:.3f} hit something, {agree:.5f} agree within {RGB_TOL}, "
          f"max diff {diff.max():.3g}, depth max diff "
          f"{np.abs(gpu['depth'][sel] - cpu['depth'][sel]).max():.3g}")
    assert hit >= min_hit_fraction
    assert agree >= AGREE_FRACTION
    for key in ("acc", "depth"):
        d = np.abs(gpu[key][sel, 0].astype(np.float64) - cpu[key][sel, 0])
        assert float(np.mean(d <= 1e-4 + 1e-4 * np.abs(cpu[key][sel, 0]))) >= AGREE_FRACTION, key


@pytest.mark.parametrize("case", ["benchmark_distribution", "dense"])
def test_trace_matches_oracle(case):
    if case == "benchmark_distribution":
        inputs, v, t = make_case(4000, 0.35, (-3.2, 0.4))
    else:  # many disks per ray: several 16-hit trace steps
        inputs, v, t = make_case(3000, 0.15, (-2.6, 0.3), seed=3)
    with NativeRendererContext(0) as ctx:
        gpu = gpu_trace(ctx, inputs, v, t, use_others=False)
    cpu = cpu_trace(inputs, v, t)
    compare(gpu, cpu)


def test_trace_second_bounce_with_auxiliary_channels():
    inputs, v, t = make_case(3000, 0.25, (-2.8, 0.4), seed=5)
    kw = dict(use_others=True, max_trace_depth=1, specular_threshold=0.05)
    with NativeRendererContext(0) as ctx:
        gpu = gpu_trace(ctx, inputs, v, t, **kw)
    cpu = cpu_trace(inputs, v, t, **kw)
    compare(gpu, cpu)
    second = cpu["mid"][:, 16 + 3:16 + 6]  # ray direction of the second trace
    assert float(np.mean(np.abs(second).sum(1) > 0)) > 0.05  # the bounce happened
    d = np.abs(gpu["aux"].astype(np.float64) - cpu["aux"]).max(1)
    assert float(np.mean(d <= 1e-5)) >= AGREE_FRACTION


def test_trace_start_from_first():
    inputs, v, t = make_case(2500, 0.3, (-3.0, 0.4), seed=7)
    with NativeRendererContext(0) as ctx:
        gpu = gpu_trace(ctx, inputs, v, t, use_others=False, start_from_first=True)
    cpu = cpu_trace(inputs, v, t, start_from_first=True)
    compare(gpu, cpu, min_hit_fraction=0.0)


def test_trace_benchmark_group_sample():
    """The 200k reflective Gaussians of the benchmark scene, all rays traced
    on the GPU, 1500 of them checked against the oracle."""
    g = scenes.make_scene("standard_1m")["reflection"]
    cam = scenes.orbit_camera("standard_1m", 0)
    center = dev(scenes.standard_camera_center(cam))
    xyz, rot_raw = dev(g["xyz"]), dev(g["rotation"])
    scale = ops.precise_exp(dev(g["scaling"]))
    rot = ops.precise_reflection_prefix(rot_raw)
    packed = ops.precise_reflection_suffix(xyz, center, rot[:, :, 2].contiguous())
    inputs = {
        "ray_origins": packed[:, 12:15].contiguous(), "ray_directions": packed[:, 9:12].contiguous(),
        "background": torch.zeros(3, device="cuda"), "means3d": xyz, "shs": dev(scenes.sh_features(g)),
        "others": torch.zeros((xyz.shape[0], 2), device="cuda"), "opacities": ops.precise_sigmoid(dev(g["opacity"])),
        "scales": scale, "rotations": ops.precise_normalize4(rot_raw), "viewmatrix": dev(cam.world_view()),
        "projmatrix": dev(cam.full_proj()), "camera_position": center,
    }
    v, t = ops.gaussian_disks(xyz, rot_raw, scale)
    with NativeRendererContext(0) as ctx:
        gpu = gpu_trace(ctx, inputs, v, t, use_others=False)
    ids = np.random.default_rng(0).choice(xyz.shape[0], 1500, replace=False)
    cpu = cpu_trace(inputs, v, t, ray_ids=ids)
    compare(gpu, cpu, ids=ids, min_hit_fraction=0.0)


def test_trace_entry_points_behave_like_the_reference():
    inputs, v, t = make_case(500, 0.3, (-3.0, 0.4))
    with NativeRendererContext(0) as ctx:
        with pytest.raises(NativeRasterizerError) as info:
            ops.trace_reflection(*inputs.values(), degree=3, context=ctx)
        assert info.value.status == 1 and "not built" in str(info.value)
        stats = ctx.optix_workspace_stats()
        assert stats["scene_ready"] == 0 and stats["gas_build_count"] == 0
        bad = t.clone()
        bad[3, 1] = v.shape[0]  # a vertex index past the end
        with pytest.raises(NativeRasterizerError) as info:
            ops.build_trace_scene(v, bad, scene_signature=3, context=ctx)
        assert info.value.status == 1
        assert ops.build_trace_scene(v, t, scene_signature=3, context=ctx) == 0
        assert ops.build_trace_scene(v, t, scene_signature=3, rebuild=False, context=ctx) == 0  # cached
        stats = ctx.optix_workspace_stats()
        assert stats["scene_ready"] == 1 and stats["gas_build_count"] == 1 and stats["scene_signature"] == 3
        assert stats["gas_output_bytes"] > 0 and stats["pipeline_create_count"] == 1
        ops.build_trace_scene(v, t, scene_signature=4, rebuild=False, context=ctx)  # new signature: rebuilt
        assert ctx.optix_workspace_stats()["gas_build_count"] == 2
        first = ops.trace_reflection(*inputs.values(), degree=3, context=ctx)
        again = ops.trace_reflection(*inputs.values(), degree=3, context=ctx)
        torch.cuda.synchronize()
        for a, b in zip(first, again):
            assert torch.equal(a, b)  # deterministic
        with pytest.raises(NativeRasterizerError) as info:
            ops.trace_reflection(*inputs.values(), degree=3, max_trace_depth=0, specular_threshold=0.0,
                                 context=ctx, use_others=True, scale_modifier=-1.0)
        assert info.value.status == 3
        ctx.release_optix_scene()
        assert ctx.optix_workspace_stats()["scene_ready"] == 0
        with pytest.raises(NativeRasterizerError):
            ops.trace_reflection(*inputs.values(), degree=3, context=ctx)
