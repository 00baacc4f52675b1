"""One standard view in one call (hs_b200_standard_view_v2).

The entry runs the session's per-view sequence (render_hybridsplat_view,
renderer.py:232-341; postprocess_raster, math.py:426-463) on one stream with
the postprocess's camera terms on a side stream. Every output must equal the
same steps called one by one through the single-purpose entry points (which
the other GPU tests check against the oracle): bit for bit, except the
per-Gaussian raster weights, which are float atomic sums and are compared to
rounding.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from hybridsplat_jittor_render_b200 import NativeRasterizerError, NativeRendererContext, ops, scenes

pytestmark = pytest.mark.gpu


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def make_view(spec, cam, *, empty_reflection=False, sh_degree=3, empty_base=False):
    scene = scenes.make_scene(spec)
    b, r = scene["base"], scene["reflection"]
    if empty_reflection:
        r = {k: v[:0] for k, v in r.items()}
    if empty_base:
        b = {k: v[:0] for k, v in b.items()}
    base = {"means3d": dev(b["xyz"]), "opacities": ops.precise_sigmoid(dev(b["opacity"])),
            "scales": ops.precise_exp(dev(b["scaling"])), "rotations": ops.precise_normalize4(dev(b["rotation"])),
            "specular": ops.precise_sigmoid(dev(b["specular"])), "roughness": ops.precise_sigmoid(dev(b["roughness"])),
            "sh": dev(scenes.sh_features(b)[:, :(sh_degree + 1) ** 2]).transpose(1, 2).contiguous()}
    nr = r["xyz"].shape[0]
    rgb = np.random.default_rng(5).random((nr, 3), dtype=np.float32)
    refl = {"means3d": dev(r["xyz"]), "opacities": ops.precise_sigmoid(dev(r["opacity"])),
            "scales": ops.precise_exp(dev(r["scaling"])), "rotations": ops.precise_normalize4(dev(r["rotation"])),
            "rotations_raw": dev(r["rotation"]), "specular": ops.precise_sigmoid(dev(r["specular"])),
            "roughness": ops.precise_sigmoid(dev(r["roughness"])), "rgb": dev(rgb)}
    trace = {"background": torch.zeros(3, device="cuda"), "shs": dev(scenes.sh_features(r)),
             "others": torch.cat([refl["specular"], refl["roughness"]], 1).contiguous(), "degree": 3,
             "use_others": False}
    camera = {"viewmatrix": dev(cam.world_view()), "projmatrix": dev(cam.full_proj()),
              "camera_position": dev(scenes.standard_camera_center(cam)), "background": torch.zeros(5, device="cuda")}
    return base, refl, trace, camera


def step_by_step(base, refl, trace, camera, cam, ctx, ctx_r, traced, depth_ratio, sh_degree=3):
    view, proj, center, bg = (camera[k] for k in ("viewmatrix", "projmatrix", "camera_position", "background"))
    colors = ops.precise_sh_colors5(base["sh"], base["means3d"], center, base["specular"], base["roughness"],
                                    sh_degree)
    rot = ops.precise_reflection_prefix(refl["rotations_raw"])
    normal = rot[:, :, 2].contiguous()
    rays = ops.precise_reflection_suffix(refl["means3d"], center, normal)
    traced_out = None
    rgb = refl["rgb"]
    if traced:
        traced_out = ops.trace_reflection(rays[:, 12:15].contiguous(), rays[:, 9:12].contiguous(), trace["background"],
                                          refl["means3d"], trace["shs"], trace["others"], refl["opacities"],
                                          refl["scales"], refl["rotations"], view, proj, center, degree=3,
                                          use_others=False, context=ctx_r)
        rgb = traced_out.rgb
    refl_colors = torch.cat([rgb, refl["specular"], refl["roughness"]], 1).contiguous()
    common = dict(viewmatrix=view, projmatrix=proj, camera_position=center, width=cam.width, height=cam.height,
                  scale_modifier=1.0, tan_fovx=cam.tan_fovx, tan_fovy=cam.tan_fovy)
    b_out = ops.rasterize_forward(bg, base["means3d"], colors, base["opacities"], base["scales"], base["rotations"],
                                  context=ctx, **common)
    r_out = ops.rasterize_forward(bg, refl["means3d"], refl_colors, refl["opacities"], refl["scales"],
                                  refl["rotations"], context=ctx_r, **common)
    fused = ops.precise_fuse_maps_planar(b_out.color[:3], r_out.color[:3], b_out.color[3:4])
    fov_x, fov_y = 2.0 * math.atan(cam.tan_fovx), 2.0 * math.atan(cam.tan_fovy)
    terms = ops.postprocess_camera_rays(cam.width, cam.height, fov_x, fov_y, view, context=ctx)
    maps = ops.standard_postprocess(b_out.color, b_out.auxiliary, terms["rays"], terms["origin"],
                                    terms["normal_rotation"], depth_ratio=depth_ratio)
    return dict(base=b_out, reflection=r_out, base_colors=colors, reflection_colors=refl_colors, rotation=rot,
                normal=normal, rays=rays, trace=traced_out, fused=fused, terms=terms, maps=maps)


def bits(a, b, what):
    a, b = a.detach().cpu().numpy(), b.detach().cpu().numpy()
    assert a.shape == b.shape, what
    if a.dtype.kind == "f":
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), what
    else:
        assert np.array_equal(a, b), what


def check(one, ref):
    for name in ("base", "reflection"):
        got, want = getattr(one, name), ref[name]
        for field in ("color", "auxiliary", "radii", "rendered"):
            bits(getattr(got, field), getattr(want, field), f"{name}.{field}")
        np.testing.assert_allclose(got.weight.cpu().numpy(), want.weight.cpu().numpy(), rtol=1e-5, atol=1e-7)
    bits(one.base_colors, ref["base_colors"], "base colours")
    bits(one.reflection_colors, ref["reflection_colors"], "reflection colours")
    bits(one.reflection_rotation, ref["rotation"], "reflection rotation")
    bits(one.reflection_normal, ref["normal"], "reflection normal")
    bits(one.reflection_rays, ref["rays"], "reflection rays")
    if ref["trace"] is not None:
        bits(one.ray_origins, ref["rays"][:, 12:15], "ray origins")
        bits(one.ray_directions, ref["rays"][:, 9:12], "ray directions")
        for field in ops.TraceOutputs._fields:
            bits(getattr(one.trace, field), getattr(ref["trace"], field), f"trace.{field}")
    for k in ref["fused"]:
        bits(one.fused[k], ref["fused"][k], k)
    for k in ("inverse_intrinsics", "rotation", "origin", "normal_rotation", "rays"):
        bits(one.camera[k], ref["terms"][k], k)
    for k in ops.STANDARD_MAPS:
        bits(one.maps[k], ref["maps"][k], k)


def run_view(spec, cam, *, traced, depth_ratio=0.0, empty_reflection=False, torch_stream=None, sh_degree=3,
             empty_base=False):
    base, refl, trace, camera = make_view(spec, cam, empty_reflection=empty_reflection, sh_degree=sh_degree,
                                          empty_base=empty_base)
    with NativeRendererContext(0) as ctx, NativeRendererContext(0) as ctx_r:
        if traced and refl["means3d"].shape[0] != 0:
            v, t = ops.gaussian_disks(refl["means3d"], refl["rotations_raw"], refl["scales"])
            ops.build_trace_scene(v, t, scene_signature=1, context=ctx_r)
        ref = step_by_step(base, refl, trace, camera, cam, ctx, ctx_r, traced, depth_ratio, sh_degree)
        torch.cuda.synchronize()
        fov_x, fov_y = 2.0 * math.atan(cam.tan_fovx), 2.0 * math.atan(cam.tan_fovy)
        stream = torch_stream or torch.cuda.current_stream()
        with torch.cuda.stream(stream):
            one = ops.standard_view(base, refl, camera["viewmatrix"], camera["projmatrix"],
                                    camera["camera_position"], camera["background"], width=cam.width,
                                    height=cam.height, tan_fovx=cam.tan_fovx, tan_fovy=cam.tan_fovy,
                                    sh_degree=sh_degree,
                                    base_context=ctx, reflection_context=ctx_r, trace=trace if traced else None,
                                    postprocess={"fov_x": fov_x, "fov_y": fov_y, "depth_ratio": depth_ratio},
                                    stream=stream.cuda_stream if torch_stream is not None else None)
        torch.cuda.synchronize()
        check(one, ref)
        return one


SMALL = scenes.SceneSpec("view_small", scenes.GroupSpec(3000), scenes.GroupSpec(600), 160, 120, 150.0)


@pytest.mark.parametrize("traced", [False, True])
@pytest.mark.parametrize("depth_ratio", [0.0, 0.5])
def test_view_matches_the_steps(traced, depth_ratio):
    run_view(SMALL, scenes.generic_camera(SMALL, 1), traced=traced, depth_ratio=depth_ratio)


@pytest.mark.parametrize("sh_degree", [0, 1, 2])
def test_view_with_lower_sh_degrees(sh_degree):
    """Fewer than 16 SH coefficients take the two-launch prologue (the fused
    grid needs 16 aligned coefficients); the outputs are the same steps'."""
    run_view(SMALL, scenes.generic_camera(SMALL, 4), traced=False, sh_degree=sh_degree)


def test_view_on_a_torch_stream():
    run_view(SMALL, scenes.generic_camera(SMALL, 3), traced=True, torch_stream=torch.cuda.Stream())


def test_view_with_no_reflective_gaussians():
    one = run_view(SMALL, scenes.generic_camera(SMALL, 2), traced=False, empty_reflection=True)
    assert one.trace is None and one.reflection_rays.shape == (0, 36)
    assert int(one.reflection.rendered[0]) == 0


@pytest.mark.parametrize("empty_reflection", [False, True])
def test_view_with_no_base_gaussians(empty_reflection):
    """An empty base group (and both groups empty): the rasters write the
    background, the prologue takes its two-launch form, the maps follow."""
    one = run_view(SMALL, scenes.generic_camera(SMALL, 5), traced=False, empty_base=True,
                   empty_reflection=empty_reflection)
    assert one.base_colors.shape == (0, 5) and int(one.base.rendered[0]) == 0


def test_view_benchmark_frame():
    """The benchmark frame: 1M base and 200k reflective Gaussians at
    1292x839, orbit view 0, reflection colours traced."""
    cam = scenes.orbit_camera("standard_1m", 0)
    run_view("standard_1m", cam, traced=True)


def test_view_needs_a_built_scene_and_two_contexts():
    cam = scenes.generic_camera(SMALL, 1)
    base, refl, trace, camera = make_view(SMALL, cam)
    args = (base, refl, camera["viewmatrix"], camera["projmatrix"], camera["camera_position"], camera["background"])
    kw = dict(width=cam.width, height=cam.height, tan_fovx=cam.tan_fovx, tan_fovy=cam.tan_fovy, sh_degree=3)
    with NativeRendererContext(0) as ctx, NativeRendererContext(0) as ctx_r:
        with pytest.raises(ValueError, match="two distinct contexts"):
            ops.standard_view(*args, base_context=ctx, reflection_context=ctx, **kw)
        with pytest.raises(NativeRasterizerError, match="OptiX scene is not built"):
            ops.standard_view(*args, base_context=ctx, reflection_context=ctx_r, trace=trace, **kw)
        # the context stays usable
        ops.standard_view(*args, base_context=ctx, reflection_context=ctx_r, **kw)
        torch.cuda.synchronize()


# ---------------------------------------------------------------- FlashGS views


def make_flashgs_view(spec, cam, *, empty_reflection=False):
    scene = scenes.make_scene(spec)
    b, r = scene["base"], scene["reflection"]
    if empty_reflection:
        r = {k: v[:0] for k, v in r.items()}
    nb, nr = b["xyz"].shape[0], r["xyz"].shape[0]

    def flashgs_inputs(g, n, colors):
        prep = ops.flashgs_prepare_host(g["opacity"], g["scaling"], g["rotation"], g["specular"], g["roughness"])
        return {"positions": dev(g["xyz"]), "shs": dev(scenes.sh_features(g).reshape(n, 48)), "colors": dev(colors),
                "opacities": dev(prep["opacity"]), "covariance": dev(prep["covariance"]),
                "scales": dev(prep["scaling"]), "rotations": dev(prep["rotation"]),
                "specular": dev(prep["specular"]), "roughness": dev(prep["roughness"])}

    cam_args = dict(width=cam.width, height=cam.height, camera_position=cam.flashgs_position,
                    camera_rotation=cam.flashgs_rotation9, focal_x=cam.fx, focal_y=cam.fy)
    rgb = np.random.default_rng(6).random((nr, 3), dtype=np.float32)
    base = dict(flashgs_inputs(b, nb, np.zeros((nb, 3), np.float32)), **cam_args)
    refl = dict(flashgs_inputs(r, nr, rgb), **cam_args)
    # the standard-activated reflection group the session traces
    group = {"means3d": dev(r["xyz"]), "rotations_raw": dev(r["rotation"]),
             "opacities": ops.precise_sigmoid(dev(r["opacity"])), "scales": ops.precise_exp(dev(r["scaling"])),
             "rotations": ops.precise_normalize4(dev(r["rotation"]))}
    others = torch.cat([ops.precise_sigmoid(dev(r["specular"])), ops.precise_sigmoid(dev(r["roughness"]))],
                       1).contiguous()
    trace = {"background": torch.zeros(3, device="cuda"), "shs": dev(scenes.sh_features(r)), "others": others,
             "degree": 3, "use_others": False}
    camera = {"world_view": dev(cam.world_view()), "full_proj": dev(cam.full_proj()),
              "camera_center": dev(scenes.standard_camera_center(cam))}
    return base, refl, group, trace, camera


def flashgs_steps(base, refl, group, trace, camera, ctx, ctx_r, traced):
    view, proj, center = camera["world_view"], camera["full_proj"], camera["camera_center"]
    b_out = ops.flashgs_forward(**base, use_sh=True, context=ctx)
    rot = ops.precise_reflection_prefix(group["rotations_raw"])
    normal = rot[:, :, 2].contiguous()
    rays = ops.precise_reflection_suffix(group["means3d"], center, normal)
    traced_out = None
    refl = dict(refl)
    if traced:
        traced_out = ops.trace_reflection(rays[:, 12:15].contiguous(), rays[:, 9:12].contiguous(), trace["background"],
                                          group["means3d"], trace["shs"], trace["others"], group["opacities"],
                                          group["scales"], group["rotations"], view, proj, center, degree=3,
                                          use_others=False, context=ctx_r)
        refl["colors"] = traced_out.rgb
    r_out = ops.flashgs_forward(**refl, use_sh=False, context=ctx_r)
    fused = ops.precise_fuse_maps_planar(b_out.color, r_out.color, b_out.other[0:1].contiguous())
    maps = ops.flashgs_postprocess(b_out, view[:3, :3].t().contiguous())
    return dict(base=b_out, reflection=r_out, rotation=rot, normal=normal, rays=rays, trace=traced_out,
                fused=fused, maps=maps)


def run_flashgs_view(spec, cam, *, traced, empty_reflection=False, torch_stream=None):
    base, refl, group, trace, camera = make_flashgs_view(spec, cam, empty_reflection=empty_reflection)
    with NativeRendererContext(0) as ctx, NativeRendererContext(0) as ctx_r:
        if traced:
            v, t = ops.gaussian_disks(group["means3d"], group["rotations_raw"], group["scales"])
            ops.build_trace_scene(v, t, scene_signature=1, context=ctx_r)
        ref = flashgs_steps(base, refl, group, trace, camera, ctx, ctx_r, traced)
        torch.cuda.synchronize()
        stream = torch_stream or torch.cuda.current_stream()
        with torch.cuda.stream(stream):
            one = ops.flashgs_view(base, refl, group, camera["world_view"], camera["full_proj"],
                                   camera["camera_center"], base_context=ctx, reflection_context=ctx_r,
                                   trace=trace if traced else None, postprocess=True,
                                   stream=stream.cuda_stream if torch_stream is not None else None)
        torch.cuda.synchronize()
    for name in ("base", "reflection"):
        for field in ops.FlashgsOutputs._fields:
            bits(getattr(getattr(one, name), field), getattr(ref[name], field), f"{name}.{field}")
    bits(one.reflection_rotation, ref["rotation"], "reflection rotation")
    bits(one.reflection_normal, ref["normal"], "reflection normal")
    bits(one.reflection_rays, ref["rays"], "reflection rays")
    if traced:
        bits(one.ray_origins, ref["rays"][:, 12:15], "ray origins")
        bits(one.ray_directions, ref["rays"][:, 9:12], "ray directions")
        for field in ops.TraceOutputs._fields:
            bits(getattr(one.trace, field), getattr(ref["trace"], field), f"trace.{field}")
    for k in ref["fused"]:
        bits(one.fused[k], ref["fused"][k], k)
    for k in ops.FLASHGS_MAPS:
        bits(one.maps[k], ref["maps"][k], k)
    return one


@pytest.mark.parametrize("traced", [False, True])
def test_flashgs_view_matches_the_steps(traced):
    run_flashgs_view(SMALL, scenes.generic_camera(SMALL, 1), traced=traced)


def test_flashgs_view_on_a_torch_stream():
    run_flashgs_view(SMALL, scenes.generic_camera(SMALL, 3), traced=True, torch_stream=torch.cuda.Stream())


def test_flashgs_view_with_no_reflective_gaussians():
    one = run_flashgs_view(SMALL, scenes.generic_camera(SMALL, 2), traced=False, empty_reflection=True)
    assert one.reflection_rays.shape == (0, 36) and int(one.reflection.rendered[0]) == 0


def test_flashgs_view_benchmark_frame():
    """The FlashGS benchmark frame (1M + 200k, 1292x839, orbit view 7),
    reflection colours traced."""
    run_flashgs_view("flashgs_1m", scenes.orbit_camera("flashgs_1m", 7), traced=True)


def test_view_records_the_raster_begin_event():
    """The optional event of the one-view entries is recorded between the
    binning and the renderers: after the view's first kernel and before its
    last."""
    cam = scenes.generic_camera(SMALL, 1)
    base, refl, trace, camera = make_view(SMALL, cam)
    with NativeRendererContext(0) as ctx, NativeRendererContext(0) as ctx_r:
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        raster = torch.cuda.Event(enable_timing=True)
        start.record()
        ops.standard_view(base, refl, camera["viewmatrix"], camera["projmatrix"], camera["camera_position"],
                          camera["background"], width=cam.width, height=cam.height, tan_fovx=cam.tan_fovx,
                          tan_fovy=cam.tan_fovy, sh_degree=3, base_context=ctx, reflection_context=ctx_r,
                          raster_begin_event=raster)
        end.record()
        torch.cuda.synchronize()
        assert raster.query()
        assert 0.0 <= start.elapsed_time(raster) <= start.elapsed_time(end)
