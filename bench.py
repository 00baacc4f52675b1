#!/usr/bin/env python
"""HybridSplat forward-renderer benchmark on B200.

One step = one full HybridSplat view of the benchmark scene (1M base + 200k
reflection Gaussians, 1292x839, fx=fy=1000, camera on the radius-4 orbit)
with inputs resident in HBM:
  standard backend (default, the configuration the metric is quoted on):
    base colours (view direction + degree-3 SH), base five-channel raster,
    reflection-ray generation (prefix + suffix), reflection raster, fusion;
  flashgs backend (--backend flashgs):
    base FlashGS raster (SH), reflection-ray generation, reflection FlashGS
    raster, fusion.
The reflection trace is not part of the headline step (the reference runs
it on OptiX and times it separately; its rebuild here cannot trace): there
its [P,3] colour output is a fixed synthetic input of the reflection raster.
The trace is timed on its own (`stages_ms.trace`, `stages_ms.trace_scene_build`)
and in `blocks.view_with_trace`, the whole view with the traced colours
feeding the reflection raster (this library's CUDA BVH tracer behind the
reference's hs_optix_* entry points).

A step is one library call per view (hs_b200_standard_view_v2 or
hs_b200_flashgs_view_v2, the same steps in the same order); --no-view-entry
issues them as the session's separate calls instead. The headline frames and
the end-to-end pass run on a stream of their own, with the camera written into one device buffer and the
standard view's outputs written into three sets used in turn, so that the
standard view entry replays each set's captured graph
(hs_b200_view_graph_stats_v1, `view_graphs` in the line); --no-view-graphs
queues every view directly.

Both steps end with the session's raw-map postprocess of the base raster
(standard: camera matrices and TF32 pixel rays on a side stream beside the
rasters, then the fused maps kernel with the surface normals; FlashGS: its
maps kernel); the reference rebuild's frame has no postprocess (the
reference's is Jittor code).

Output: one JSON line on rank 0 (driver contract). `value` is whole-job
frames per second with device-resident inputs, the median over repeated
timed loops of exactly --steps steps each; `e2e` adds the per-frame
host->device camera upload and the device->host read of the eight maps the
session fetches (rgb, acc, dpt, norm, surf_norm, spec, diffuse and
reflection rgb).
`blocks` carries the other benchmark configurations measured by the same
run: the FlashGS 20-view orbit (`flashgs`), the 6M + 1M 1920x1080 scene
view-sharded over the GPUs (`large_6m`) and the 3840x2160 stress frame split
into tile-row strips across the GPUs (`stress_4k`), each with the reference
CUDA backend rebuilt for sm_100 on one GPU beside it.

--impl reference times the reference's CPU-side path as restated by the CPU
oracle (the reference has no CPU renderer) on the same workload, one full
frame per step.
Multi-GPU (torchrun, N>1): one process per GPU; the scene is broadcast once
from rank 0 into every rank's device buffers through the library's NCCL
communicator; every rank renders its own orbit views (weak scaling) or its
own strip of one frame (strong scaling); no collective runs inside a timed
region; per-step times are the max over ranks.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from dataclasses import dataclass
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

METRIC = "FPS @1292x839, 1M base+200k refl Gaussians, 1/2/4/8 B200; per-stage ms"


@dataclass(frozen=True)
class Workload:
    scene: str
    metric: str
    sharding: str  # "view-sharded" (weak scaling) or "tile-strip" (strong scaling)


WORKLOADS = {
    "view": Workload("standard_1m", METRIC, "view-sharded"),
    "large_6m": Workload("large_6m", "FPS @1920x1080, 6M base+1M refl Gaussians, 160-view orbit, view-sharded",
                         "view-sharded"),
    "stress_4k": Workload("stress_4k", "frames/s of one 3840x2160 frame, 3M base+500k refl (inflated scales), "
                          "tile-strip sharded", "tile-strip"),
}
SM_COUNT = 148
# Algorithmic FP32 work of one pixel x Gaussian blend evaluation, counted
# from the blend functions (FMA = 2 flop; each IEEE division and expf = 1):
# standard (csrc/standard_math.cuh blend): 39 flop up to the alpha < 1/255
# exit, 76 for an evaluation that blends; FlashGS (csrc/flashgs_math.cuh
# blend) always blends: 75.
FLOP_STANDARD_DEAD = 39
FLOP_STANDARD_LIVE = 76
FLOP_FLASHGS = 75
# Timed loops: each times exactly --steps steps; loops repeat until both
# bounds are met and the median loop is reported.
HEADLINE_MIN_SECONDS, HEADLINE_MIN_REPEATS = 3.0, 10
BLOCK_MIN_SECONDS, BLOCK_MIN_REPEATS = 1.0, 5
MAX_REPEATS = 2000
VIEW_OUTPUT_SETS = 3


def parse_args():
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--sequential", action="store_true",
                   help="render the two raster branches one after the other (v1 calls) instead of concurrently")
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--backend", choices=("standard", "flashgs"), default="standard")
    p.add_argument("--workload", choices=tuple(WORKLOADS), default="view")
    p.add_argument("--no-cpu-baseline", action="store_true", help="skip the timed CPU oracle leg")
    p.add_argument("--no-reference-gpu", action="store_true", help="skip timing the reference CUDA rebuild")
    p.add_argument("--no-blocks", action="store_true",
                   help="skip the flashgs / large_6m / stress_4k blocks of the default run")
    p.add_argument("--readback", choices=("at-raster", "after-call", "before-call"), default="after-call",
                   help="e2e: queue frame s-1's map read-back before or after frame s's raster calls, or after "
                        "them to start when frame s's renderers may start (one-call views)")
    p.add_argument("--scale", type=float, default=1.0, help="Gaussian-count scale (profiling runs only)")
    p.add_argument("--profile-frames", type=int, default=0,
                   help="render this many frames untimed and exit (a short, fixed launch sequence for ncu)")
    p.add_argument("--profile-reference", action="store_true",
                   help="with --profile-frames: render with the reference CUDA rebuild (oracle/_ref)")
    p.add_argument("--trace", action="store_true",
                   help="with --profile-frames: trace the reflection colours of every frame")
    p.add_argument("--profile-replays", action="store_true",
                   help="with --profile-frames: render the frames on a stream of their own with the output sets in "
                        "turn, as the headline loop does (standard views replayed from their third use of a set on)")
    p.add_argument("--no-view-entry", action="store_true",
                   help="standard views as the session's separate calls instead of hs_b200_standard_view_v2")
    p.add_argument("--no-view-graphs", action="store_true",
                   help="queue every standard view directly (HS_B200_VIEW_GRAPHS=0): no captured graph replays")
    return p.parse_args()


def emit(line: dict):
    print(json.dumps(line), flush=True)


def scene_counts(name: str, scale: float) -> tuple[int, int]:
    from hybridsplat_jittor_render_b200 import scenes
    spec = scenes.SCENES[name]
    return (max(1, int(round(spec.base.count * scale))), max(1, int(round(spec.reflection.count * scale))))


def workload_config(workload: Workload, backend: str, scale: float, world: int) -> dict:
    """The `config` of a bench line; both arms print the same dict."""
    from hybridsplat_jittor_render_b200 import scenes
    spec = scenes.SCENES[workload.scene]
    nb, nr = scene_counts(workload.scene, scale)
    what = (f"one {spec.width}x{spec.height} frame per step, tile rows split across the GPUs"
            if workload.sharding == "tile-strip" else f"one {spec.width}x{spec.height} orbit view per step per GPU")
    return {"workload": f"{backend} backend, {nb} base + {nr} reflection Gaussians, {what}",
            "scene": workload.scene, "backend": backend, "gaussians": [nb, nr],
            "resolution": [spec.width, spec.height], "parallelism": f"{workload.sharding} x{world}",
            "l2": "inputs larger than L2"}


def reflection_trace_rgb(count: int) -> np.ndarray:
    """Synthetic stand-in for the OptiX trace colour of the reflection Gaussians."""
    rng = np.random.default_rng(99)
    return rng.random((count, 3), dtype=np.float32)


# --------------------------------------------------------------------------- multi-rank plumbing

class Job:
    """This process's rank: device, NCCL communicator (library), max over ranks."""

    def __init__(self):
        import torch
        from hybridsplat_jittor_render_b200 import multigpu
        info = multigpu.rank_info()
        self.rank, self.world, self.local_rank = info.rank, info.world_size, info.local_rank
        torch.cuda.set_device(self.local_rank)
        self.device = torch.device("cuda", self.local_rank)
        self.comm = multigpu.communicator(self.local_rank, timeout_s=300.0)

    @property
    def is_root(self) -> bool:
        return self.rank == 0

    def barrier(self):
        self.comm.barrier()

    def max(self, *values: float) -> list[float]:
        return self.comm.allreduce_max(list(values))

    def close(self):
        self.comm.close()


SCENE_FIELDS = (("xyz", 3), ("features_dc", 3), ("features_rest", 45), ("scaling", 2), ("rotation", 4),
                ("opacity", 1), ("specular", 1), ("roughness", 1))
FLASHGS_FIELDS = (("opacity", 1), ("covariance", 6), ("scaling", 2), ("rotation", 4), ("specular", 1),
                  ("roughness", 1))


def scene_layout(name: str, scale: float, flashgs: bool):
    from hybridsplat_jittor_render_b200 import multigpu
    shapes = []
    for group, n in zip(("base", "reflection"), scene_counts(name, scale)):
        shapes += [(f"{group}/{f}", (n, w)) for f, w in SCENE_FIELDS]
        if flashgs:
            shapes += [(f"{group}/fg_{f}", (n, w)) for f, w in FLASHGS_FIELDS]
    shapes.append(("reflection/trace_rgb", (scene_counts(name, scale)[1], 3)))
    return multigpu.PackedLayout.of(shapes)


class DeviceScene:
    """The scene's arrays in one device buffer, filled on rank 0 from the
    seeded generator (plus the FlashGS host activation when asked for) and
    broadcast once to every rank; `host` keeps rank 0's numpy copy."""

    def __init__(self, job: Job, name: str, scale: float, flashgs: bool):
        import torch
        from hybridsplat_jittor_render_b200 import ops, scenes
        self.name = name
        self.counts = scene_counts(name, scale)
        layout = scene_layout(name, scale, flashgs)
        self.flat = torch.empty(layout.total, dtype=torch.float32, device=job.device)
        self.host = None
        if job.is_root:
            raw = scenes.make_scene(name, scale=scale)
            arrays = {}
            for group in ("base", "reflection"):
                g = raw[group]
                n = g["xyz"].shape[0]
                for f, w in SCENE_FIELDS:
                    arrays[f"{group}/{f}"] = g[f].reshape(n, w)
                if flashgs:
                    pr = ops.flashgs_prepare_host(g["opacity"], g["scaling"], g["rotation"], g["specular"],
                                                  g["roughness"])
                    for f, w in FLASHGS_FIELDS:
                        arrays[f"{group}/fg_{f}"] = pr[f].reshape(n, w)
            arrays["reflection/trace_rgb"] = reflection_trace_rgb(self.counts[1])
            staging = torch.empty(layout.total, dtype=torch.float32, pin_memory=True)
            layout.pack(arrays, staging.numpy())
            self.flat.copy_(staging, non_blocking=True)
            torch.cuda.current_stream().synchronize()
            self.host = raw
        job.comm.broadcast_buffer(self.flat, stream=torch.cuda.current_stream().cuda_stream)
        self.views = layout.views(self.flat)

    def group(self, group: str) -> dict:
        pre = group + "/"
        return {k[len(pre):]: v for k, v in self.views.items() if k.startswith(pre)}


# --------------------------------------------------------------------------- the view

class Frame:
    """Device-resident state and the per-view render sequence."""

    def __init__(self, scene: DeviceScene, backend: str, device, library=None, concurrent: bool = True):
        import torch
        from hybridsplat_jittor_render_b200 import NativeRendererContext, ops, scenes
        self.torch, self.ops, self.scenes = torch, ops, scenes
        self.backend, self.device, self.library = backend, device, library
        self.ctx = NativeRendererContext(device.index or 0, library=library)
        # Concurrent branches (hs_b200_*_forward_many_v2) need a context each;
        # sequential ones share one, as the reference session does.
        self.concurrent = concurrent
        self.ctx_r = NativeRendererContext(device.index or 0, library=library) if concurrent else self.ctx
        b, r = scene.group("base"), scene.group("reflection")
        self.nb, self.nr = scene.counts

        def sh16(g):  # [P, 16, 3], DC first
            return torch.cat([g["features_dc"].view(-1, 1, 3), g["features_rest"].view(-1, 15, 3)], 1)

        # session-init activation (not timed)
        self.r_xyz, self.r_rot_raw = r["xyz"], r["rotation"]
        self.r_spec = ops.precise_sigmoid(r["specular"], library=library)
        self.r_rough = ops.precise_sigmoid(r["roughness"], library=library)
        self.trace_rgb = r["trace_rgb"]
        if backend == "standard":
            self.b_xyz = b["xyz"]
            self.b_sh = sh16(b).transpose(1, 2).contiguous()
            self.b_spec = ops.precise_sigmoid(b["specular"], library=library)
            self.b_rough = ops.precise_sigmoid(b["roughness"], library=library)
            self.b_op = ops.precise_sigmoid(b["opacity"], library=library)
            self.b_scale = ops.precise_exp(b["scaling"], library=library)
            self.b_rot = ops.precise_normalize4(b["rotation"], library=library)
            self.r_op = ops.precise_sigmoid(r["opacity"], library=library)
            self.r_scale = ops.precise_exp(r["scaling"], library=library)
            self.r_rot = ops.precise_normalize4(self.r_rot_raw, library=library)
            self.r_colors = torch.cat([self.trace_rgb, self.r_spec, self.r_rough], 1).contiguous()
            self.bg5 = torch.zeros(5, device=device)
        else:
            def prep(g, colors):
                n = g["xyz"].shape[0]
                return [g["xyz"], sh16(g).reshape(n, 48).contiguous(), colors, g["fg_opacity"], g["fg_covariance"],
                        g["fg_scaling"], g["fg_rotation"], g["fg_specular"], g["fg_roughness"]]
            self.b_in = prep(b, torch.zeros((self.nb, 3), device=device))
            self.r_in = prep(r, self.trace_rgb)
        # This library fuses the view's glue (direction + SH + concatenation,
        # transposes + fusion); a library with only the reference ABI runs the
        # reference session's sequence.
        lib = library if library is not None else ops.load_native_library()
        self.fused_glue = hasattr(lib, "hs_b200_precise_sh_colors5_f32_v1")
        # The session's raw-map postprocess is part of the frame with this
        # library (the reference's is Jittor code, which its rebuild lacks):
        # the camera terms and pixel rays on a side stream beside the rasters,
        # then one maps kernel after them.
        self.with_post = hasattr(lib, "hs_b200_postprocess_camera_f32_v1")
        self.post_stream = torch.cuda.Stream(device=device) if self.with_post else None
        self.cam_terms_buf = self.rays_buf = None
        self.cam = None
        self.split = None  # list: per raster call stage timings (instrumented pass)
        self.tile_rows = None  # (begin, end): render only this strip of tile rows
        self.r_scene = r
        self.traced = False  # render() traces the reflection colours (enable_trace)
        # Views go to the library as one call (hs_b200_standard_view_v2,
        # hs_b200_flashgs_view_v2) unless instrumented, rendered in strips or
        # run sequentially.
        self.view_entry = hasattr(lib, f"hs_b200_{backend}_view_v2")
        self.raster_event = None  # one-call views record it when their renderers may start
        # the standard view's outputs and its camera row on the device: three
        # sets used in turn (next_slot: the set of the next view); a set is
        # rewritten only after its read-back is queued
        self.view_outs = [None] * VIEW_OUTPUT_SETS
        self.cam_slots = [None] * VIEW_OUTPUT_SETS
        self.cam_dev = None
        self.next_slot = 0

    def enable_trace(self) -> float:
        """Builds the reflection trace scene of the session (the disks of the
        reflective Gaussians, hs_optix_build_scene_v1) and makes every view
        trace its reflection colours. Returns the build's device ms."""
        torch, ops = self.torch, self.ops
        r = self.r_scene
        self.r_scale_exp = ops.precise_exp(r["scaling"])
        self.r_rot_unit = ops.precise_normalize4(self.r_rot_raw)
        self.r_sh16 = torch.cat([r["features_dc"].view(-1, 1, 3), r["features_rest"].view(-1, 15, 3)], 1).contiguous()
        self.r_op_act = ops.precise_sigmoid(r["opacity"])
        self.r_others = torch.cat([self.r_spec, self.r_rough], 1).contiguous()
        self.bg3 = torch.zeros(3, device=self.device)
        vertices, triangles = ops.gaussian_disks(self.r_xyz, self.r_rot_raw, self.r_scale_exp)
        torch.cuda.synchronize()
        times = []
        for signature in range(1, 5):  # the first build also allocates the scene's buffers
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            ops.build_trace_scene(vertices, triangles, scene_signature=signature, context=self.ctx_r)
            e1.record()
            torch.cuda.synchronize()
            times.append(e0.elapsed_time(e1))
        self.traced = True
        self.trace_first_build_ms = times[0]
        return float(np.median(times[1:]))

    def trace(self, rays):
        """The reflection trace of one view (hs_optix_trace_f32_v1): one ray
        per reflective Gaussian from the prepared reflection rays."""
        ops = self.ops
        view, proj = self.view, self.proj
        return ops.trace_reflection(rays[:, 12:15].contiguous(), rays[:, 9:12].contiguous(), self.bg3, self.r_xyz,
                                    self.r_sh16, self.r_others, self.r_op_act, self.r_scale_exp, self.r_rot_unit,
                                    view, proj, self.center, degree=3, use_others=False, context=self.ctx_r)

    def close(self):
        self.ctx.close()
        if self.ctx_r is not self.ctx:
            self.ctx_r.close()

    def camera_buffer(self, slot: int, like):
        """The device camera row of output set `slot` (allocated like `like`)."""
        buf = self.cam_slots[slot]
        if buf is None or buf.shape != like.shape:
            buf = self.cam_slots[slot] = self.torch.empty(like.shape, dtype=like.dtype, device=self.device)
        return buf

    def set_camera(self, cam, upload_from=None, uploaded=False):
        """Per-view camera state: the row (view and projection matrices,
        centre) in the camera buffer of the next view's output set, copied
        from `upload_from` (pinned host or device memory) or from the camera
        on the current stream, or (uploaded) already written there."""
        torch = self.torch
        self.cam = cam
        host = upload_from if upload_from is not None else torch.from_numpy(camera_row(cam, self.scenes))
        buf = self.camera_buffer(self.next_slot, host)
        if not uploaded:
            buf.copy_(host, non_blocking=True)
        self.cam_dev = buf
        self.view, self.proj, self.center = buf[:16].view(4, 4), buf[16:32].view(4, 4), buf[32:35]
        # FlashGS takes the camera as host values; the device row gives the
        # ray centre and the postprocess's normal rotation

    def render(self, events=None):
        """One view. `events`, when given, is a list of CUDA events recorded
        between the stages (base, reflection prepare, reflection, fusion, and
        with the postprocess its camera terms and its maps: 5 or 7 events); the
        branches then run one after the other so that each stage is timed
        alone. Otherwise, with self.concurrent, both raster branches go to the
        library in one concurrent call, and the postprocess's camera terms and
        pixel rays run on a side stream beside them."""
        ops, torch, cam, lib = self.ops, self.torch, self.cam, self.library
        sequential = events is not None or not self.concurrent
        if self.one_call(events):
            return self.render_one_call()
        rec = (lambda i: events[i].record()) if events else (lambda i: None)
        post = self.with_post
        terms = None
        fov_x, fov_y = 2.0 * math.atan(cam.tan_fovx), 2.0 * math.atan(cam.tan_fovy)
        if post and self.backend == "standard" and self.cam_terms_buf is None:
            f = dict(dtype=torch.float32, device=self.device)
            self.cam_terms_buf = torch.empty(30, **f)
            self.rays_buf = torch.empty((cam.height * cam.width, 3), **f)
        if post and self.backend == "standard" and events is None:
            self.post_stream.wait_stream(torch.cuda.current_stream(self.device))
            terms = ops.postprocess_camera_rays(cam.width, cam.height, fov_x, fov_y, self.view, context=self.ctx,
                                                stream=self.post_stream.cuda_stream, camera=self.cam_terms_buf,
                                                rays=self.rays_buf)
        rec(0)
        if self.backend == "standard":
            if self.fused_glue:
                colors = ops.precise_sh_colors5(self.b_sh, self.b_xyz, self.center, self.b_spec, self.b_rough, 3,
                                                library=lib)
            else:
                d = ops.precise_direction(self.b_xyz, self.center, library=lib)
                rgb = ops.precise_sh_to_rgb(self.b_sh, d, 3, library=lib)
                colors = torch.cat([rgb, self.b_spec, self.b_rough], 1)
            common = dict(viewmatrix=self.view, projmatrix=self.proj, camera_position=self.center, width=cam.width,
                          height=cam.height, scale_modifier=1.0, tan_fovx=cam.tan_fovx, tan_fovy=cam.tan_fovy,
                          tile_rows=self.tile_rows)
            base_call = dict(background=self.bg5, means3d=self.b_xyz, colors=colors, opacities=self.b_op,
                             scales=self.b_scale, rotations=self.b_rot, context=self.ctx, **common)
            refl_call = dict(background=self.bg5, means3d=self.r_xyz, colors=self.r_colors, opacities=self.r_op,
                             scales=self.r_scale, rotations=self.r_rot, context=self.ctx_r, **common)
            single, many = ops.rasterize_forward, ops.rasterize_forward_many
        else:
            common = dict(width=cam.width, height=cam.height, camera_position=cam.flashgs_position,
                          camera_rotation=cam.flashgs_rotation9, focal_x=cam.fx, focal_y=cam.fy,
                          initial_pair_capacity=2_000_000, tile_rows=self.tile_rows)
            names = ("positions", "shs", "colors", "opacities", "covariance", "scales", "rotations", "specular",
                     "roughness")
            base_call = dict(zip(names, self.b_in), use_sh=True, context=self.ctx, **common)
            refl_call = dict(zip(names, self.r_in), use_sh=False, context=self.ctx_r, **common)
            single, many = ops.flashgs_forward, ops.flashgs_forward_many
        center = self.center
        if sequential:
            base = single(**base_call)
            rec(1)
            if self.split is not None:
                self.split.append(("base", self.ctx.read_stage_timing()))
        rot = ops.precise_reflection_prefix(self.r_rot_raw, library=lib)
        normal_raw = rot[:, :, 2].contiguous()
        rays = ops.precise_reflection_suffix(self.r_xyz, center, normal_raw, library=lib)
        if self.traced:
            # the traced colours feed the reflection raster, as in the session
            traced = self.trace(rays).rgb
            if self.backend == "standard":
                refl_call["colors"] = torch.cat([traced, self.r_spec, self.r_rough], 1).contiguous()
            else:
                refl_call["colors"] = traced
        rec(2)
        if sequential:
            refl = single(**refl_call)
            if self.split is not None:
                self.split.append(("reflection", self.ctx_r.read_stage_timing()))
        else:
            base, refl = many([base_call, refl_call], stream=torch.cuda.current_stream(self.device).cuda_stream)
        if self.backend == "standard":
            base_rgb, spec = base.color[:3], base.color[3:4]
        else:
            base_rgb, spec = base.color, base.other[0:1]
        rec(3)
        if self.fused_glue:
            fused = ops.precise_fuse_maps_planar(base_rgb, refl.color[:3], spec, library=lib)
        else:
            fused = ops.precise_fuse_maps(base_rgb.permute(1, 2, 0).contiguous(),
                                          refl.color[:3].permute(1, 2, 0).contiguous(),
                                          spec.permute(1, 2, 0).contiguous(), library=lib)
        rec(4)
        maps = None
        if post:
            if self.backend == "standard":
                if terms is None:  # instrumented pass: the camera terms alone, on this stream
                    terms = ops.postprocess_camera_rays(cam.width, cam.height, fov_x, fov_y, self.view,
                                                        context=self.ctx, camera=self.cam_terms_buf,
                                                        rays=self.rays_buf)
                else:
                    torch.cuda.current_stream(self.device).wait_stream(self.post_stream)
                rec(5)
                maps = ops.standard_postprocess(base.color, base.auxiliary, terms["rays"], terms["origin"],
                                                terms["normal_rotation"], library=lib)
            else:
                normal_rotation = self.view[:3, :3].t().contiguous()
                rec(5)
                maps = ops.flashgs_postprocess(base, normal_rotation, library=lib)
            rec(6)
        return base, refl, fused, rays, maps

    def one_call(self, events=None) -> bool:
        return self.view_entry and events is None and self.concurrent and self.tile_rows is None

    def render_one_call(self):
        """The whole view as one library call (ops.standard_view,
        ops.flashgs_view): the same steps as render(), in the same order, on
        the current stream (standard: the camera terms on the library's side
        stream)."""
        torch, cam = self.torch, self.cam
        if self.backend == "flashgs":
            common = dict(width=cam.width, height=cam.height, camera_position=cam.flashgs_position,
                          camera_rotation=cam.flashgs_rotation9, focal_x=cam.fx, focal_y=cam.fy,
                          initial_pair_capacity=2_000_000)
            names = ("positions", "shs", "colors", "opacities", "covariance", "scales", "rotations", "specular",
                     "roughness")
            group = dict(means3d=self.r_xyz, rotations_raw=self.r_rot_raw)
            trace = None
            if self.traced:
                group.update(opacities=self.r_op_act, scales=self.r_scale_exp, rotations=self.r_rot_unit)
                trace = dict(background=self.bg3, shs=self.r_sh16, others=self.r_others, degree=3, use_others=False)
            out = self.ops.flashgs_view(dict(zip(names, self.b_in), **common), dict(zip(names, self.r_in), **common),
                                        group, self.view, self.proj, self.center, base_context=self.ctx,
                                        reflection_context=self.ctx_r, trace=trace, postprocess=self.with_post,
                                        stream=torch.cuda.current_stream(self.device).cuda_stream,
                                        raster_begin_event=self.raster_event)
            return out.base, out.reflection, out.fused, out.reflection_rays, out.maps
        base = dict(means3d=self.b_xyz, opacities=self.b_op, scales=self.b_scale, rotations=self.b_rot,
                    specular=self.b_spec, roughness=self.b_rough, sh=self.b_sh)
        refl = dict(means3d=self.r_xyz, opacities=self.r_op, scales=self.r_scale, rotations=self.r_rot,
                    rotations_raw=self.r_rot_raw, specular=self.r_spec, roughness=self.r_rough, rgb=self.trace_rgb)
        trace = (dict(background=self.bg3, shs=self.r_sh16, others=self.r_others, degree=3, use_others=False)
                 if self.traced else None)
        post = None
        if self.with_post:
            post = {"fov_x": 2.0 * math.atan(cam.tan_fovx), "fov_y": 2.0 * math.atan(cam.tan_fovy),
                    "depth_ratio": 0.0}
        slot = self.next_slot
        self.next_slot = (slot + 1) % VIEW_OUTPUT_SETS
        reuse = self.view_outs[slot]
        if reuse is not None and (reuse.trace is None) != (trace is None):
            reuse = None
        out = self.ops.standard_view(base, refl, self.view, self.proj, self.center, self.bg5, width=cam.width,
                                     height=cam.height, tan_fovx=cam.tan_fovx, tan_fovy=cam.tan_fovy, sh_degree=3,
                                     base_context=self.ctx, reflection_context=self.ctx_r, trace=trace,
                                     postprocess=post,
                                     stream=torch.cuda.current_stream(self.device).cuda_stream,
                                     raster_begin_event=self.raster_event, out=reuse)
        self.view_outs[slot] = out
        return out.base, out.reflection, out.fused, out.reflection_rays, out.maps

    def maps_for_host(self, result):
        """The maps the session reads back (session.py:33-42): rgb, acc, dpt,
        norm, surf_norm, spec, diffuse and reflection rgb, with the
        postprocess; without it (the reference rebuild) the raw planes they
        come from (no surface normals)."""
        base, _, fused, _, maps = result
        if maps is not None:
            return [fused["rgb_map"], maps["acc_map"], maps["dpt_map"], maps["norm_map"], maps["surf_norm_map"],
                    maps["spec_map"], fused["dif_rgb_map"], fused["ref_rgb_map"]]
        if self.backend == "standard":
            acc, depth, normal, spec = base.auxiliary[1], base.auxiliary[0], base.auxiliary[2:5], base.color[3]
        else:
            acc, depth, normal, spec = base.alpha[0], base.depth[0], base.normal, base.other[0]
        return [fused["rgb_map"], acc, depth, normal, spec, fused["dif_rgb_map"], fused["ref_rgb_map"]]

    def launches_per_step(self, width: int, height: int, replayed: bool = False) -> int:
        """Kernels of this library launched by one render() call (memsets and
        copies excluded; `replayed`: the standard view replayed as a captured
        graph, whose two totals publications are one status kernel): per raster
        call preprocess, totals publication, the
        depth sort, pair offsets, emission, the tile sort, ranges, tile order
        (which also publishes the wait status) and the rasteriser; plus the
        elementwise kernels of the view. A sort of n items in p 8-bit passes
        launches 1 histogram + p one-sweep passes, or 3 kernels per pass
        (count, scan, scatter) from 2^21 items. The tile sorts' pair counts
        are the groups' `rendered` counts of the last view, an upper bound of
        the pairs emitted after culling (the same side of 2^21 on the
        benchmark frame: 4.5M / 3.66M base, under 1M reflection)."""
        torch = self.torch
        if getattr(self, "pair_counts", None) is None:
            base, refl = self.render()[:2]
            torch.cuda.synchronize()
            self.pair_counts = (int(base.rendered.reshape(-1)[0]), int(refl.rendered.reshape(-1)[0]))

        def sort_launches(n: int, bits: int) -> int:
            passes = math.ceil(bits / 8)
            return 0 if n == 0 else (3 * passes if n >= 1 << 21 else 1 + passes)

        tiles = ((width + 15) // 16) * ((height + 15) // 16)
        tile_bits = max(1, int(tiles).bit_length())
        per_raster = 0
        for points, pairs in zip((self.nb, self.nr), self.pair_counts):
            per_raster += 1 + 1 + sort_launches(points, 32) + 1 + 1 + sort_launches(pairs, tile_bits) + 1 + 1 + 1
        if self.fused_glue:
            extra = 1 if self.backend == "standard" else 0  # direction + SH + concatenation
        else:
            extra = 2 if self.backend == "standard" else 0  # direction + SH
        if self.with_post:
            # standard: camera inputs, 2 inverse transposes, camera pack, pixel
            # rays, maps (the inverses' cuSOLVER/cuBLAS kernels are not ours);
            # FlashGS: maps
            extra += 6 if self.backend == "standard" else 1
        if self.one_call():
            # the one-call entries prepare the reflection in one kernel (prefix,
            # normal column, suffix and the standard colours), which the
            # standard entry runs in the same grid as the base colours; a
            # traced standard view concatenates its colours after the trace
            if self.backend == "standard":
                extra -= 1 if self.traced else 2
            else:
                extra -= 1
            if self.with_post:
                extra -= 1  # the maps kernel also does the fusion
        if replayed:
            per_raster -= 1
        return per_raster + extra + 3  # + reflection prefix, suffix, fusion


def camera_row(cam, scenes) -> np.ndarray:
    return np.concatenate([cam.world_view().reshape(-1), cam.full_proj().reshape(-1),
                           scenes.standard_camera_center(cam)]).astype(np.float32)


# --------------------------------------------------------------------------- clocks

class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        import torch
        # nvidia-smi numbers GPUs physically; select ours by UUID so that
        # CUDA_VISIBLE_DEVICES remapping does not matter.
        self.index = f"GPU-{torch.cuda.get_device_properties(device_index).uuid}"
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (FileNotFoundError, OSError):
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        if self.path is None or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9 and parts[1].replace(".", "").isdigit():
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": float(rows[0][2]), "reasons": reasons,
                "samples": len(rows), "power_w_max": max(float(r[3]) for r in rows if r[3].replace(".", "").isdigit())}


# --------------------------------------------------------------------------- CPU oracle

def cpu_oracle_frame(scene_np, name: str, backend: str, row_stride: int, threads: int) -> dict:
    """Times the CPU oracle on orbit view 0 of scene `name`, sampling every
    `row_stride`-th tile row (1: the whole frame); returns the frame time
    (blending and binning of the sampled rows scaled by row_stride) and, per
    Gaussian group, the blend evaluations by the reference's rule and those
    that changed a pixel."""
    from hybridsplat_jittor_render_b200 import ops, scenes
    from oracle import oracle
    cam = scenes.orbit_camera(name, 0)
    total_ms = 0.0
    evals, live = {}, {}
    t0 = time.perf_counter()
    for gname in ("base", "reflection"):
        g = scene_np[gname]
        n = g["xyz"].shape[0]
        trace = reflection_trace_rgb(scene_np["reflection"]["xyz"].shape[0])
        stats = np.zeros(5, np.float64)
        if backend == "standard":
            center = scenes.standard_camera_center(cam)
            if gname == "base":
                d = oracle.precise_direction(g["xyz"], center)
                rgb = oracle.precise_sh_to_rgb(np.ascontiguousarray(scenes.sh_features(g).transpose(0, 2, 1)), d, 3)
            else:
                rgb = trace
            colors = np.concatenate([rgb, oracle.precise_sigmoid(g["specular"]), oracle.precise_sigmoid(g["roughness"])], 1)
            inputs = {"background": np.zeros(5, np.float32), "means3d": g["xyz"], "colors": colors,
                      "opacities": oracle.precise_sigmoid(g["opacity"]), "scales": oracle.precise_exp(g["scaling"]),
                      "rotations": oracle.precise_normalize4(g["rotation"]), "viewmatrix": cam.world_view(),
                      "projmatrix": cam.full_proj()}
            oracle.standard_forward(inputs, width=cam.width, height=cam.height, threads=threads,
                                    row_stride=row_stride, stage_ms=stats)
        else:
            pr = ops.flashgs_prepare_host(g["opacity"], g["scaling"], g["rotation"], g["specular"], g["roughness"])
            inputs = {"positions": g["xyz"], "shs": scenes.sh_features(g).reshape(n, 48),
                      "colors": trace if gname == "reflection" else np.zeros((n, 3), np.float32),
                      "opacities": pr["opacity"], "covariance": pr["covariance"], "scales": pr["scaling"],
                      "rotations": pr["rotation"], "specular": pr["specular"], "roughness": pr["roughness"]}
            oracle.flashgs_forward(inputs, width=cam.width, height=cam.height, use_sh=gname == "base",
                                   camera_position=cam.flashgs_position, camera_rotation=cam.flashgs_rotation9,
                                   focal_x=cam.fx, focal_y=cam.fy, threads=threads, row_stride=row_stride,
                                   stage_ms=stats)
        # preprocess covers every Gaussian; binning and blending cover 1/row_stride of the tile rows
        total_ms += stats[0] + row_stride * (stats[1] + stats[2])
        evals[gname] = row_stride * stats[3]
        live[gname] = row_stride * stats[4]
    wall = time.perf_counter() - t0
    return {"frame_ms": total_ms, "evaluations": evals, "live": live, "wall_s": wall}


# --------------------------------------------------------------------------- reference arm

def run_reference_arm(args, workload: Workload) -> int:
    """The reference's CPU path on the host cores: the reference has no CPU
    renderer, so each step renders one full frame (base + reflection, every
    tile row) with the CPU oracle's restatement of the reference kernels, on
    all host threads. Rank 0 only."""
    from hybridsplat_jittor_render_b200 import scenes
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if int(os.environ.get("RANK", "0")) != 0:
        return 0
    threads = len(os.sched_getaffinity(0))
    scene = scenes.make_scene(workload.scene, scale=args.scale)
    for _ in range(min(1, max(0, args.warmup))):
        cpu_oracle_frame(scene, workload.scene, args.backend, 1, threads)
    times = [cpu_oracle_frame(scene, workload.scene, args.backend, 1, threads)["frame_ms"]
             for _ in range(max(1, args.steps))]
    ms = float(np.median(times))
    fps = 1000.0 / ms
    sample = (f"one full {args.backend} frame (base + reflection, all tile rows) per step by the CPU oracle "
              f"(the reference has no CPU renderer; the oracle restates its kernels), {threads} threads, "
              f"median of {len(times)} steps after {min(1, max(0, args.warmup))} warm-up frame")
    emit({"metric": workload.metric, "value": fps, "unit": "frames/s", "n_gpus": world, "steps": args.steps,
          "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
          "scaling": "strong" if workload.sharding == "tile-strip" else "weak",
          "vs_baseline": None, "dtype": "f32", "data": "synthetic",
          "config": workload_config(workload, args.backend, args.scale, world),
          "impl": "reference",
          "cpu_baseline": {"value": fps, "unit": "frames/s", "cores": threads, "kind": "port", "sample": sample},
          "e2e": {"value": fps, "unit": "frames/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}})
    return 0


# --------------------------------------------------------------------------- timing helpers

def views_for(job: Job, name: str, sharding: str, steps: int, warmup: int) -> list[int]:
    from hybridsplat_jittor_render_b200 import scenes
    if sharding == "tile-strip":
        return [0] * (warmup + steps)
    n_views = max(scenes.SCENES[name].views, 20)
    return [(job.rank + job.world * s) % n_views for s in range(warmup + steps)]


def prime(frame: Frame, cams, warmup: int, device_cams):
    """Session priming: one untimed render of each distinct view sizes the
    grow-only workspaces (as a long-running session would), then the
    warm-up steps."""
    for cam in {id(c): c for c in cams}.values():
        frame.set_camera(cam)
        frame.render()
    for s in range(warmup):
        frame.set_camera(cams[s], upload_from=device_cams[s])
        frame.render()
    frame.torch.cuda.synchronize()


def timed_loops(job: Job, frame: Frame, cams, device_cams, warmup: int, steps: int, min_seconds: float,
                min_repeats: int) -> dict:
    """Repeats a timed loop of exactly `steps` steps (CUDA events on the
    launching stream, synchronised on both sides, after a barrier) until
    min_seconds and min_repeats are reached; returns the per-step ms of the
    median loop, max over ranks."""
    torch = frame.torch
    stream = torch.cuda.current_stream()

    def one_loop():
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for s in range(steps):
            frame.set_camera(cams[warmup + s], upload_from=device_cams[warmup + s])
            frame.render()
        end.record(stream)
        return start, end

    torch.cuda.synchronize()
    s0, e0 = one_loop()
    torch.cuda.synchronize()
    first = s0.elapsed_time(e0)
    repeats = int(min(MAX_REPEATS, max(min_repeats, math.ceil(min_seconds * 1000.0 / max(first, 1e-3)))))
    repeats = int(job.max(float(repeats))[0])  # every rank runs the same number of loops
    job.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    events = [one_loop() for _ in range(repeats)]
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    job.barrier()
    loops = [a.elapsed_time(b) / steps for a, b in events]
    median = float(statistics.median(loops))
    worst = job.max(median)[0]
    return {"ms_per_step": worst, "repeats": repeats, "loop_ms_min": min(loops) * steps,
            "loop_ms_max": max(loops) * steps, "timed_wall_s": wall}


def stage_split(frame: Frame, cam, steps: int) -> dict:
    """Per-stage ms (instrumented pass, not the headline): CUDA events between
    the frame's stages plus the library's own stage events inside each raster
    call, the branches sequential."""
    torch = frame.torch
    stage_names = ("base_raster", "reflection_prepare", "reflection_raster", "fusion")
    if frame.with_post:
        stage_names += ("postprocess_camera_rays", "postprocess_maps")
    n = len(stage_names)
    sums = np.zeros(n)
    for c in {id(c): c for c in (frame.ctx, frame.ctx_r)}.values():
        c.stage_timing(True)
        c.read_stage_timing()
    # one untimed pass first: the one-call frames before it never launched some
    # of the separate steps' kernels, and a first launch loads its module
    frame.set_camera(cam)
    frame.render([torch.cuda.Event(enable_timing=True) for _ in range(n + 1)])
    torch.cuda.synchronize()
    for c in {id(c): c for c in (frame.ctx, frame.ctx_r)}.values():
        c.read_stage_timing()
    frame.split = []
    for _ in range(steps):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(n + 1)]
        frame.set_camera(cam)
        frame.render(ev)
        torch.cuda.synchronize()
        sums += [ev[i].elapsed_time(ev[i + 1]) for i in range(n)]
    for c in {id(c): c for c in (frame.ctx, frame.ctx_r)}.values():
        c.stage_timing(False)
    split, frame.split = frame.split, None
    stages = {k: float(v / steps) for k, v in zip(stage_names, sums)}
    for group in ("base", "reflection"):
        runs = [t for g, t in split if g == group]
        for k in ("preprocess_ms", "binning_ms", "blend_ms"):
            stages[f"{group}_{k}"] = float(np.mean([t[k] for t in runs]))
    return stages


def reference_rebuild(scene: DeviceScene, backend: str, device, cams, warmup: int, steps: int):
    """The reference's own CUDA backend compiled for sm_100 from its sources
    (oracle/_ref), same frames (whole frames: the reference has no strip
    entry point), same device inputs, branches sequential as in the
    reference session, one GPU; None when the rebuild is absent."""
    import torch
    ref_path = REPO / "oracle" / "_ref" / "libref_hybridsplat.so"
    if not ref_path.exists():
        return None
    from hybridsplat_jittor_render_b200.native_runtime import bind_library
    ref = bind_library(ref_path, require_optix=False)
    rframe = Frame(scene, backend, device, library=ref, concurrent=False)
    for cam in {id(c): c for c in cams}.values():
        rframe.set_camera(cam)
        rframe.render()
    for s in range(warmup):
        rframe.set_camera(cams[s])
        rframe.render()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for s in range(steps):
        rframe.set_camera(cams[warmup + s])
        rframe.render()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    rframe.close()
    return {"value": 1000.0 / ms, "unit": "frames/s", "ms_per_step": ms,
            "what": "the reference's own CUDA backend compiled for sm_100 from its sources (oracle/_ref), "
                    "same frames, same device inputs, one GPU"}


# --------------------------------------------------------------------------- blocks

def run_block(job: Job, args, scene: DeviceScene, workload: Workload, backend: str) -> dict:
    """One further benchmark configuration in the same run: timed loops,
    stage split on view 0 and (one GPU) the reference rebuild beside it."""
    import torch
    from hybridsplat_jittor_render_b200 import multigpu, scenes
    spec = scenes.SCENES[workload.scene]
    frame = Frame(scene, backend, job.device, concurrent=not args.sequential)
    frame.view_entry &= not args.no_view_entry
    strips = workload.sharding == "tile-strip"
    if strips:
        frame.tile_rows = multigpu.tile_strips((spec.height + 15) // 16, job.world)[job.rank]
    views = views_for(job, workload.scene, workload.sharding, args.steps, args.warmup)
    cams = [scenes.orbit_camera(workload.scene, v) for v in views]
    device_cams = [torch.from_numpy(camera_row(c, scenes)).to(job.device) for c in cams]
    prime(frame, cams, args.warmup, device_cams)
    job.barrier()
    t = timed_loops(job, frame, cams, device_cams, args.warmup, args.steps, BLOCK_MIN_SECONDS, BLOCK_MIN_REPEATS)
    ms = t["ms_per_step"]
    out = {"metric": workload.metric, "value": (1 if strips else job.world) * 1000.0 / ms, "unit": "frames/s",
           "ms_per_step": ms, "steps": args.steps, "warmup": args.warmup, "repeats": t["repeats"],
           "scaling": "strong" if strips else "weak",
           "config": workload_config(workload, backend, args.scale, job.world)}
    if job.world == 1:
        out["stages_ms"] = stage_split(frame, scenes.orbit_camera(workload.scene, 0), min(args.steps, 10))
        frame.close()
        if not args.no_reference_gpu:
            ref = reference_rebuild(scene, backend, job.device, cams, args.warmup, args.steps)
            if ref is not None:
                ref["ratio"] = ref["ms_per_step"] / ms
                out["reference_cuda_rebuild"] = ref
    else:
        frame.close()
    torch.cuda.synchronize()
    return out


# --------------------------------------------------------------------------- our arm

def run_ours(args, workload: Workload) -> int:
    import torch
    if args.no_view_graphs:
        os.environ["HS_B200_VIEW_GRAPHS"] = "0"
    job = Job()
    return run_headline(job, args, workload)


def run_headline(job, args, workload: Workload) -> int:
    import torch
    from hybridsplat_jittor_render_b200 import multigpu, scenes

    device = job.device
    world = job.world
    spec = scenes.SCENES[workload.scene]
    strips = workload.sharding == "tile-strip"
    blocks_on = not args.no_blocks and workload.scene == "standard_1m" and args.profile_frames == 0
    scene = DeviceScene(job, workload.scene, args.scale,
                        flashgs=args.backend == "flashgs" or (blocks_on and workload.scene == "standard_1m"))
    library = None
    if args.profile_frames > 0 and args.profile_reference:
        from hybridsplat_jittor_render_b200.native_runtime import bind_library
        library = bind_library(REPO / "oracle" / "_ref" / "libref_hybridsplat.so", require_optix=False)
    frame = Frame(scene, args.backend, device, library=library, concurrent=not args.sequential)
    frame.view_entry &= not args.no_view_entry
    if strips:
        frame.tile_rows = multigpu.tile_strips((spec.height + 15) // 16, world)[job.rank]
    views = views_for(job, workload.scene, workload.sharding, args.steps, args.warmup)
    cams = [scenes.orbit_camera(workload.scene, v) for v in views]
    if args.profile_frames > 0:
        if args.trace:
            frame.enable_trace()
        torch.cuda.synchronize()
        with torch.cuda.stream(torch.cuda.Stream(device=device) if args.profile_replays
                               else torch.cuda.current_stream(device)):
            for s in range(args.profile_frames):
                frame.set_camera(cams[s % len(cams)])
                frame.render()
        torch.cuda.synchronize()
        if args.profile_replays and frame.one_call() and args.backend == "standard":
            print(json.dumps({"view_graphs": frame.ops.view_graph_stats(frame.ctx)}), flush=True)
        job.close()
        return 0

    # The per-view camera values of every step, resident on the device before
    # the timed region like the scene (the end-to-end pass below uploads them
    # from pinned host memory instead).
    cam_rows = [torch.from_numpy(camera_row(c, scenes)) for c in cams]
    device_cams = [row.to(device) for row in cam_rows]
    # The headline frames and the end-to-end pass run on a stream of their
    # own (a graph capture needs a stream other than the legacy default
    # stream); the instrumented passes and the other blocks stay on the
    # legacy default stream, where the separate calls and their events run.
    work = torch.cuda.Stream(device=device)
    torch.cuda.synchronize()
    with torch.cuda.stream(work):
        prime(frame, cams, args.warmup, device_cams)
        job.barrier()
        with ClockSampler(job.local_rank) as clocks:
            t = timed_loops(job, frame, cams, device_cams, args.warmup, args.steps, HEADLINE_MIN_SECONDS,
                            HEADLINE_MIN_REPEATS)
    torch.cuda.synchronize()
    ms = t["ms_per_step"]
    fps_total = (1 if strips else world) * 1000.0 / ms

    stages = stage_split(frame, scenes.orbit_camera(workload.scene, 0), args.steps)

    torch.cuda.synchronize()
    with torch.cuda.stream(work):
        e2e = end_to_end(job, frame, cams, cam_rows, args)
    torch.cuda.synchronize()

    line = None
    if job.is_root:
        line = {"metric": workload.metric, "value": fps_total, "unit": "frames/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
                "scaling": "strong" if strips else "weak",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded scene with the benchmark "
                "configuration's sizes and distributions; fixed synthetic trace colours)",
                "config": workload_config(workload, args.backend, args.scale, world),
                "timing": {"repeats": t["repeats"], "statistic": f"median of {t['repeats']} timed loops of exactly "
                           f"{args.steps} steps, max over ranks", "loop_ms_min": t["loop_ms_min"],
                           "loop_ms_max": t["loop_ms_max"], "timed_wall_s": t["timed_wall_s"],
                           "priming": "one untimed render of each timed view before the warm-up steps",
                           "branches": "sequential v1 calls" if args.sequential else
                                       f"the whole view in one call (hs_b200_{args.backend}_view_v2: both "
                                       "rasters concurrent)" if frame.one_call() else
                                       "base and reflection rasters in one concurrent call "
                                       "(hs_b200_*_forward_many_v2)",
                           "stages_ms": "from a separate pass with the branches sequential, each stage alone; "
                                        "postprocess_camera_rays (camera matrices and the TF32 pixel rays, which "
                                        "in the headline frame run on a side stream beside the rasters) and "
                                        "postprocess_maps (the fused maps kernel after them) are part of the frame",
                           "postprocess": "in the frame (session raw-map postprocess of the base raster); the "
                                          "reference rebuild's frame has none (its postprocess is Jittor code)"},
                "stages_ms": stages, "clocks": clocks.summary(), "e2e": e2e,
                "gpu_launches": frame.launches_per_step(
                    spec.width, spec.height,
                    replayed=frame.one_call() and args.backend == "standard" and not args.no_view_graphs)
                * args.steps * t["repeats"]}
        if frame.one_call() and args.backend == "standard":
            line["view_graphs"] = dict(frame.ops.view_graph_stats(frame.ctx), enabled=not args.no_view_graphs,
                                       what="standard views replayed as captured graphs "
                                            "(hs_b200_view_graph_stats_v1 on the base context, whole run)")
    if world == 1 and line is not None:
        # single GPU: render-kernel roofline, CPU baseline, reference CUDA rebuild
        line.update(roofline_and_baselines(args, workload, frame, cams, scene, stages, line["clocks"], ms))
    traced = trace_block(job, args, frame, cams, device_cams, strips)
    if line is not None:
        stages["trace"] = traced.pop("trace_ms")
        stages["trace_scene_build"] = traced.pop("scene_build_ms")
        stages["trace_scene_first_build"] = traced.pop("scene_first_build_ms")
        line.setdefault("blocks", {})["view_with_trace"] = traced
    frame.close()
    frame = None
    torch.cuda.synchronize()

    if blocks_on:
        blocks = {}
        blocks["flashgs"] = run_block(job, args, scene, WORKLOADS["view"], "flashgs")
        blocks["flashgs"]["what"] = ("FlashGS backend, 20-view orbit of the benchmark scene (config 2): "
                                     "base FlashGS raster with SH, reflection prepare, reflection raster, fusion")
        del scene
        torch.cuda.empty_cache()
        for name in ("large_6m", "stress_4k"):
            big = DeviceScene(job, WORKLOADS[name].scene, args.scale, flashgs=False)
            blocks[name] = run_block(job, args, big, WORKLOADS[name], "standard")
            del big
            torch.cuda.empty_cache()
        if line is not None:
            line.setdefault("blocks", {}).update(blocks)
    job.barrier()
    job.close()
    if line is not None:
        emit(line)
    return 0


def trace_block(job: Job, args, frame: Frame, cams, device_cams, strips: bool) -> dict:
    """The reflection trace: the session's scene build (once), one view's
    trace timed alone (CUDA events around hs_optix_trace_f32_v1), and the
    whole view with the traced colours feeding the reflection raster."""
    import torch
    build_ms = frame.enable_trace()
    frame.set_camera(cams[0])
    rays = frame.render()[3]
    torch.cuda.synchronize()
    times = []
    for _ in range(args.steps + 2):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        frame.trace(rays)
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1))
    trace_ms = float(statistics.median(times[2:]))
    prime(frame, cams, args.warmup, device_cams)
    job.barrier()
    t = timed_loops(job, frame, cams, device_cams, args.warmup, args.steps, BLOCK_MIN_SECONDS, BLOCK_MIN_REPEATS)
    return {"value": (1 if strips else job.world) * 1000.0 / t["ms_per_step"], "unit": "frames/s",
            "ms_per_step": t["ms_per_step"], "steps": args.steps, "repeats": t["repeats"],
            "what": "the headline view plus the reflection trace (hs_optix_trace_f32_v1, CUDA BVH tracer) whose "
                    "colours feed the reflection raster, as the reference session renders a view",
            "trace_ms": trace_ms, "scene_build_ms": build_ms, "scene_first_build_ms": frame.trace_first_build_ms,
            "trace_rays": frame.nr}


def end_to_end(job: Job, frame: Frame, cams, cam_rows, args) -> dict:
    """The same frames through the public API with host buffers: every step
    uploads its camera from pinned host memory and reads the session's eight
    maps back into pinned host memory (two slots) on a copy stream."""
    import torch
    stream = torch.cuda.current_stream()
    pinned_cam = [row.pin_memory() for row in cam_rows]
    res = frame.render()
    host_maps = [[torch.empty(m.shape, dtype=m.dtype, pin_memory=True) for m in frame.maps_for_host(res)]
                 for _ in range(2)]
    d2h = sum(m.numel() * m.element_size() for m in host_maps[0])
    h2d = pinned_cam[0].numel() * 4  # the camera row: view, projection, centre
    copy_stream = torch.cuda.Stream(device=frame.device)

    at_raster = args.readback == "at-raster" and frame.one_call()
    raster_events = [torch.cuda.Event() for _ in range(2)] if at_raster else None
    # frame s writes output set s % 3 (standard view entry): after the
    # read-back of the frame that last wrote it
    copied = [torch.cuda.Event() for _ in range(VIEW_OUTPUT_SETS)]
    copy_queued = [False] * VIEW_OUTPUT_SETS
    # frame s's camera row goes to camera set s % 3 on an upload stream,
    # queued before frame s - 1 is rendered (after the frame that last read
    # that set): the upload does not wait in the frame stream's queue
    upload_stream = torch.cuda.Stream(device=frame.device)
    uploaded = [torch.cuda.Event() for _ in range(VIEW_OUTPUT_SETS)]
    rendered = [None] * VIEW_OUTPUT_SETS

    def upload(s):
        slot = s % VIEW_OUTPUT_SETS
        buf = frame.camera_buffer(slot, pinned_cam[s])
        if rendered[slot] is not None:
            upload_stream.wait_event(rendered[slot])
        with torch.cuda.stream(upload_stream):
            buf.copy_(pinned_cam[s], non_blocking=True)
        uploaded[slot].record(upload_stream)

    def read_back(s, out, done):
        copy_stream.wait_event(done)
        if at_raster:  # frame s + 1's binning is done: its renderers take the link's traffic best
            copy_stream.wait_event(raster_events[(s + 1) % 2])
        with torch.cuda.stream(copy_stream):
            for dst, src in zip(host_maps[s % 2], frame.maps_for_host(out)):
                dst.copy_(src, non_blocking=True)
                src.record_stream(copy_stream)
            copied[s % VIEW_OUTPUT_SETS].record(copy_stream)
            copy_queued[s % VIEW_OUTPUT_SETS] = True

    def run(first, count, marks=None):
        pending = None
        upload(first)
        for s in range(first, first + count):
            if args.readback == "before-call" and pending is not None:
                read_back(*pending)
                pending = None
            frame.next_slot = s % VIEW_OUTPUT_SETS
            stream.wait_event(uploaded[s % VIEW_OUTPUT_SETS])
            frame.set_camera(cams[s], upload_from=pinned_cam[s], uploaded=True)
            if s + 1 < first + count:
                upload(s + 1)
            if at_raster:
                frame.raster_event = raster_events[s % 2]
            if copy_queued[s % VIEW_OUTPUT_SETS]:
                stream.wait_event(copied[s % VIEW_OUTPUT_SETS])
            if marks is not None:
                marks.append((torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)))
                marks[-1][0].record(stream)
                host_t0 = time.perf_counter()
            out = frame.render()
            if marks is not None:
                host_ms.append((time.perf_counter() - host_t0) * 1000.0)
                marks[-1][1].record(stream)
            done = torch.cuda.Event()
            done.record(stream)
            rendered[s % VIEW_OUTPUT_SETS] = done
            if pending is not None:
                read_back(*pending)
            pending = (s, out, done)
        read_back(*pending)
        stream.wait_stream(copy_stream)
        return pending[1]

    # untimed steps of the same pipeline: the caching allocator settles the
    # blocks that the copy stream keeps alive one frame longer
    run(0, args.warmup)
    torch.cuda.synchronize()
    loops = []
    res = None
    job.barrier()
    for _ in range(5):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        res = run(args.warmup, args.steps)
        e1.record(stream)
        torch.cuda.synchronize()
        loops.append(e0.elapsed_time(e1) / args.steps)
    # one more loop, outside the statistic, with an event pair around every
    # frame: how long the frames take on the device under the read-back, and
    # the device time between them
    marks = []
    host_ms = []
    run(args.warmup, args.steps, marks)
    torch.cuda.synchronize()
    frame_ms = [a.elapsed_time(b) for a, b in marks]
    gap_ms = [marks[i][1].elapsed_time(marks[i + 1][0]) for i in range(len(marks) - 1)]
    frame.raster_event = None
    job.barrier()
    e2e_ms = job.max(float(statistics.median(loops)))[0]
    # The host-link ceiling: the same read-back alone (last frame's maps, same
    # pinned slots), on every rank at once.
    maps = frame.maps_for_host(res)
    job.barrier()
    c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(copy_stream):
        c0.record(copy_stream)
        for s in range(args.steps):
            for dst, src in zip(host_maps[s % 2], maps):
                dst.copy_(src, non_blocking=True)
        c1.record(copy_stream)
    torch.cuda.synchronize()
    d2h_ms = c0.elapsed_time(c1) / args.steps
    d2h_worst = job.max(d2h_ms)[0]
    job.barrier()
    value = job.world * 1000.0 / e2e_ms
    ceiling = job.world * 1000.0 / d2h_worst
    return {"value": value, "unit": "frames/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "overlap": ("maps of frame s-1 copied to pinned host memory on a copy stream queued before frame s's "
                        "raster calls" if args.readback == "before-call" else
                        "maps of frame s-1 copied on a copy stream once frame s's binning is done and its "
                        "renderers may start" if at_raster else
                        "maps of frame s-1 copied on a copy stream queued after frame s's raster calls return"),
            "pipeline": (f"frames on their own stream, each writing output set s % {VIEW_OUTPUT_SETS} after that "
                         "set's previous read-back; each camera row uploaded from pinned memory on an upload stream "
                         "one frame ahead; standard views replayed as captured graphs unless --no-view-graphs"),
            "statistic": "median of 5 loops of exactly --steps steps, max over ranks",
            "d2h_ms_alone": d2h_worst, "d2h_gbs_alone_per_gpu": d2h / (d2h_worst * 1e6),
            "host_link_ceiling_fps": ceiling, "fraction_of_host_link_ceiling": value / ceiling,
            "frame_ms_under_readback": float(statistics.median(frame_ms)),
            "gap_ms_between_frames": float(statistics.median(gap_ms)) if gap_ms else 0.0,
            "host_ms_per_view_call": float(statistics.median(host_ms)) if host_ms else 0.0}


def cpu_stages_block() -> dict:
    """The reference's CPU-side stages on the CPU plumbing workload (10k + 2k
    Gaussians, SH 3, 20 views): checkpoint validation, activation, the
    FlashGS host activation as shipped, both camera loaders and the camera
    matrices, median wall ms on one thread. The stages that run the
    reference's Python are read from the committed measurement (the
    reference checkout is not on this host); the rest are timed here."""
    from oracle import cpu_stages

    block = {"workload": "cpu_plumbing (10000 base + 2000 reflective Gaussians, SH degree 3, 20 views "
                         "1292x839)", "unit": "ms", "statistic": "median of 7 runs, one thread"}
    if cpu_stages.RESULTS.exists():
        committed = json.loads(cpu_stages.RESULTS.read_text())
        block["all_stages"] = {"host": committed["host"], "total_ms": committed["total_ms"],
                                   "stages_ms": {k: v["ms"] for k, v in committed["stages"].items()},
                                   "source": "oracle/cpu_stages_config0.json (" + committed["command"] + ")"}
    live = cpu_stages.host_stages(7)
    block["gpu_host"] = {"host": cpu_stages.host_info(), "stages_ms": {k: v["ms"] for k, v in live.items()},
                          "what": "stages that need no reference Python, timed live on this GPU host"}
    return block


def roofline_and_baselines(args, workload: Workload, frame: Frame, cams, scene: DeviceScene, stages: dict,
                           clocks: dict, headline_ms: float) -> dict:
    out = {}
    peaks = {}
    peak_path = REPO / "MEASURED_PEAKS.json"
    if peak_path.exists():
        peaks = json.loads(peak_path.read_text())
    threads = len(os.sched_getaffinity(0))
    cpu = None
    if not args.no_cpu_baseline and workload.scene == "standard_1m":
        cpu = cpu_oracle_frame(scene.host, workload.scene, args.backend, 1, threads)
        out["cpu_baseline"] = {"value": 1000.0 / cpu["frame_ms"], "unit": "frames/s", "cores": threads,
                               "kind": "port",
                               "sample": f"one full {args.backend} frame (base + reflection) of the benchmark "
                                         f"scene by the CPU oracle, {threads} threads, {cpu['wall_s']:.1f} s"}
    if not args.no_cpu_baseline:
        out["cpu_stages"] = cpu_stages_block()
    # Roofline of the dominant kernel: the rasteriser's launch for the base
    # group of view 0 (FP32-pipe bound). Work = the reference-rule
    # evaluations counted by the CPU oracle on the same view, split into
    # those that exit at the alpha test and those that blend; time = that
    # launch's CUDA events inside the library.
    blend_ms = stages["base_blend_ms"]
    sm_mhz = clocks.get("sm_mhz") or peaks.get("sm_max_mhz") or 1965.0
    peak_tflops = SM_COUNT * 128 * 2 * sm_mhz * 1e6 / 1e12
    traffic = None
    tpath = REPO / "profiles" / "traffic.json"
    if tpath.exists():
        traffic = json.loads(tpath.read_text()).get(f"{args.backend}_render_base_bytes_per_launch")
    if cpu is not None:
        evals = cpu["evaluations"]["base"]
        live = cpu["live"]["base"]
        if args.backend == "standard":
            flop = live * FLOP_STANDARD_LIVE + (evals - live) * FLOP_STANDARD_DEAD
        else:
            flop = evals * FLOP_FLASHGS
        achieved = flop / (blend_ms * 1e-3) / 1e12
        out["roofline"] = {"bound": "fp32", "kernel": f"{args.backend} render_kernel, base-group launch of view 0",
                           "kernel_ms": blend_ms, "achieved": achieved, "peak": peak_tflops, "unit": "TFLOP/s",
                           "frac": achieved / peak_tflops, "traffic": traffic,
                           "work": f"{evals:.4g} reference-rule evaluations ({live:.4g} blend), {flop:.4g} flop",
                           "peak_source": f"nominal FP32 FMA rate, {SM_COUNT} SMs x 128 lanes x 2 flop at "
                                          f"{sm_mhz:.0f} MHz (measured median SM clock under load); "
                                          "MEASURED_PEAKS.json has no FP32 figure"}
    if not args.no_reference_gpu:
        ref = reference_rebuild(scene, args.backend, frame.device, cams, args.warmup, args.steps)
        if ref is not None:
            ref["ratio"] = ref["ms_per_step"] / headline_ms
            out["reference_cuda_rebuild"] = ref
    return out


def main() -> int:
    args = parse_args()
    workload = WORKLOADS[args.workload]
    if args.impl == "reference":
        return run_reference_arm(args, workload)
    return run_ours(args, workload)


if __name__ == "__main__":
    sys.exit(main())
