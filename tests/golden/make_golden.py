"""Generates tests/golden/*.npz from the reference library itself.

Run on a CUDA host after `python oracle/build_ref.py` has produced
oracle/_ref/libref_hybridsplat.so (the reference's own native sources
compiled for Blackwell). For every case in cases.py it stores the inputs and
the reference outputs of:
  * hs_flashgs_forward_f32_v1 for the base (SH) and reflection (colour)
    groups, plus hs_flashgs_debug_copy_v1 (preprocess state, sorted pairs,
    tile ranges);
  * hs_rasterizer_forward_f32_v1 (standard backend) for both groups;
  * hs_flashgs_prepare_npz_host_f32_v1;
and, once, the fixed-rounding elementwise entry points on seeded inputs.

Usage: python tests/golden/make_golden.py [--out tests/golden]
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path

import numpy as np
import torch

REPO = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(Path(__file__).resolve().parent))

from cases import CASES, camera_for, raw_groups  # noqa: E402

from hybridsplat_jittor_render_b200 import native_runtime as nr  # noqa: E402
from hybridsplat_jittor_render_b200 import ops, scenes  # noqa: E402

REF_LIBRARY = REPO / "oracle" / "_ref" / "libref_hybridsplat.so"
FLASHGS_OUT = ("color", "other", "depth", "alpha", "normal", "median_depth", "distortion", "rendered")


def to_dev(a, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda:0", dtype)


def flashgs_inputs(group, lib) -> dict:
    n = group["xyz"].shape[0]
    prep = ops.flashgs_prepare_host(group["opacity"], group["scaling"], group["rotation"], group["specular"],
                                    group["roughness"], library=lib)
    return {"positions": group["xyz"], "shs": scenes.sh_features(group).reshape(n, 48),
            "colors": scenes.sigmoid(group["features_dc"][:, 0, :]), "opacities": prep["opacity"],
            "covariance": prep["covariance"], "scales": prep["scaling"], "rotations": prep["rotation"],
            "specular": prep["specular"], "roughness": prep["roughness"]}


def flashgs_case(lib, ctx, group, cam, use_sh, background):
    n = group["xyz"].shape[0]
    inputs = flashgs_inputs(group, lib)
    dev = {k: to_dev(v) for k, v in inputs.items()}
    out = ops.flashgs_forward(*dev.values(), width=cam.width, height=cam.height, use_sh=use_sh,
                              camera_position=cam.flashgs_position, camera_rotation=cam.flashgs_rotation9,
                              focal_x=cam.fx, focal_y=cam.fy, background=background,
                              initial_pair_capacity=1 << 16, context=ctx)
    torch.cuda.synchronize()
    result = {f"in_{k}": np.ascontiguousarray(v, np.float32) for k, v in inputs.items()}
    for k, v in zip(FLASHGS_OUT, out):
        result[f"out_{k}"] = v.cpu().numpy()
    if n > 0:
        for k, v in ctx.flashgs_debug_snapshot().items():
            result[f"dbg_{k}"] = v
    return result


def standard_inputs(group, cam, background, lib) -> dict:
    n = group["xyz"].shape[0]
    xyz = to_dev(group["xyz"])
    center = to_dev(scenes.standard_camera_center(cam))
    if n > 0:
        direction = ops.precise_direction(xyz, center, library=lib)
        sh = to_dev(np.ascontiguousarray(scenes.sh_features(group).transpose(0, 2, 1)))
        rgb = ops.precise_sh_to_rgb(sh, direction, 3, library=lib)
        colors = torch.cat([rgb, ops.precise_sigmoid(to_dev(group["specular"]), library=lib),
                            ops.precise_sigmoid(to_dev(group["roughness"]), library=lib)], 1).contiguous()
        opac = ops.precise_sigmoid(to_dev(group["opacity"]), library=lib)
        scales = ops.precise_exp(to_dev(group["scaling"]), library=lib)
        rots = ops.precise_normalize4(to_dev(group["rotation"]), library=lib)
    else:
        colors = torch.zeros((0, 5), device="cuda:0")
        opac = torch.zeros((0, 1), device="cuda:0")
        scales = torch.zeros((0, 2), device="cuda:0")
        rots = torch.zeros((0, 4), device="cuda:0")
    return {"background": to_dev(np.array([*background, 0.0, 0.0], np.float32)), "means3d": xyz,
            "colors": colors, "opacities": opac, "scales": scales, "rotations": rots,
            "viewmatrix": to_dev(cam.world_view()), "projmatrix": to_dev(cam.full_proj()),
            "camera_position": center}


def standard_case(lib, ctx, group, cam, background):
    inputs = standard_inputs(group, cam, background, lib)
    out = ops.rasterize_forward(*inputs.values(), width=cam.width, height=cam.height, scale_modifier=1.0,
                                tan_fovx=cam.tan_fovx, tan_fovy=cam.tan_fovy, context=ctx)
    torch.cuda.synchronize()
    result = {f"in_{k}": v.cpu().numpy() for k, v in inputs.items()}
    for k, v in zip(("color", "auxiliary", "weight", "radii", "rendered"), out):
        result[f"out_{k}"] = v.cpu().numpy()
    return result


def precise_case(lib) -> dict:
    rng = np.random.default_rng(11)
    n = 4096
    d = {"in_x": rng.normal(0, 3, n).astype(np.float32), "in_q": rng.normal(0, 1, (n, 4)).astype(np.float32),
         "in_points": rng.normal(0, 2, (n, 3)).astype(np.float32),
         "in_center": np.array([0.3, -4.0, 1.2], np.float32),
         "in_sh": rng.normal(0, 0.3, (n, 3, 16)).astype(np.float32),
         "in_normal": rng.normal(0, 1, (n, 3)).astype(np.float32), "in_base": rng.random((n, 3)).astype(np.float32),
         "in_refl": rng.random((n, 3)).astype(np.float32), "in_spec": rng.random((n, 1)).astype(np.float32)}
    dv = {k: to_dev(v) for k, v in d.items()}
    d["out_exp"] = ops.precise_exp(dv["in_x"], library=lib).cpu().numpy()
    d["out_sigmoid"] = ops.precise_sigmoid(dv["in_x"], library=lib).cpu().numpy()
    d["out_normalize4"] = ops.precise_normalize4(dv["in_q"], library=lib).cpu().numpy()
    direction = ops.precise_direction(dv["in_points"], dv["in_center"], library=lib)
    d["out_direction"] = direction.cpu().numpy()
    for deg in range(4):
        d[f"out_sh{deg}"] = ops.precise_sh_to_rgb(dv["in_sh"], direction, deg, library=lib).cpu().numpy()
    d["out_reflection_prefix"] = ops.precise_reflection_prefix(dv["in_q"], library=lib).cpu().numpy()
    d["out_disk_rotation"] = ops.precise_disk_rotation(dv["in_q"], library=lib).cpu().numpy()
    d["out_reflection_suffix"] = ops.precise_reflection_suffix(dv["in_points"], dv["in_center"], dv["in_normal"],
                                                               library=lib).cpu().numpy()
    for k, v in ops.precise_fuse_maps(dv["in_base"], dv["in_refl"], dv["in_spec"], library=lib).items():
        d[f"out_{k}"] = v.cpu().numpy()
    return d


def main() -> int:
    parser = argparse.ArgumentParser()
    parser.add_argument("--out", type=Path, default=Path(__file__).resolve().parent)
    args = parser.parse_args()
    lib = nr.bind_library(REF_LIBRARY, require_optix=False)
    ctx = nr.NativeRendererContext(0, library=lib)
    args.out.mkdir(parents=True, exist_ok=True)
    for case in CASES:
        groups = raw_groups(case)
        cam = camera_for(case)
        data = {"camera_R": cam.R, "camera_T": cam.T, "camera_center": cam.center,
                "camera_size": np.array([cam.width, cam.height]), "camera_focal": np.array([cam.fx, cam.fy]),
                "camera_flashgs_rotation9": np.array(cam.flashgs_rotation9, np.float32),
                "camera_tan_fov": np.array([cam.tan_fovx, cam.tan_fovy], np.float64),
                "background": np.array(case.background, np.float32)}
        for gname, use_sh in (("base", True), ("reflection", False)):
            for k, v in flashgs_case(lib, ctx, groups[gname], cam, use_sh, case.background).items():
                data[f"flashgs_{gname}_{k}"] = v
            for k, v in standard_case(lib, ctx, groups[gname], cam, case.background).items():
                data[f"standard_{gname}_{k}"] = v
        np.savez_compressed(args.out / f"{case.name}.npz", **data)
        print(case.name, {k: int(v.reshape(-1)[0]) for k, v in data.items() if k.endswith("rendered")})
    np.savez_compressed(args.out / "precise.npz", **precise_case(lib))
    rng = np.random.default_rng(13)
    n = 4096
    raw = [rng.normal(0, 1.5, (n, 1)), rng.normal(-4, 0.5, (n, 2)), rng.normal(0, 1, (n, 4)),
           rng.normal(-1, 1, (n, 1)), rng.normal(0, 1, (n, 1))]
    raw = [a.astype(np.float32) for a in raw]
    prep = ops.flashgs_prepare_host(*raw, library=lib)
    np.savez_compressed(args.out / "prepare_host.npz", in_opacity=raw[0], in_scaling=raw[1], in_rotation=raw[2],
                        in_specular=raw[3], in_roughness=raw[4], **{f"out_{k}": v for k, v in prep.items()})
    ctx.close()
    print("golden fixtures written to", args.out)
    return 0


if __name__ == "__main__":
    sys.exit(main())
