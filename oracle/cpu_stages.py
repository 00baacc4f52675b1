"""CPU-side stages of the reference, timed on a host's cores (baseline only).

Test and baseline infrastructure: nothing here is on the product path. The
workload is the CPU plumbing configuration: a strict 29-member NPZ
checkpoint with 10,000 base and 2,000 reflective Gaussians at SH degree 3
(seed 0, the distributions of ``scenes.SCENES["cpu_plumbing"]``), plus the
same 20 orbit views (1292 x 839 after the loaders' quarter scaling,
fx = fy = 1000, radius 4, looking at the origin) written both as EasyVolcap
OpenCV YAML (``intri.yml``/``extri.yml``) and as FlashGS ``cameras.json``.

Stages, each the median of ``--runs`` (>= 5) wall-clock runs on one thread:

``checkpoint.infer``
    ``infer_checkpoint_contract`` with the SHA-256 pin
    (jittor_hybridsplat/checkpoint.py:151-231).
``checkpoint.validate``
    ``validate_checkpoint_archive`` (checkpoint.py:374-387): the inference
    again, the path/size/SHA re-check, the ZIP member audit with CRC test and
    the read of every array with its shape/dtype/finite checks
    (checkpoint.py:234-371).
``activation``
    a numpy float32 restatement of the lazy parameter activations of
    checkpoint.py:438-461 (exp of the scaling, safe_normalize(eps=1e-12,
    clamp) of the rotation from math.py:15-18, sigmoid of opacity, specular
    and roughness) for both groups; Jittor, which the reference uses for
    them, is not installed.
``flashgs_prepare_host``
    ``hs_flashgs_prepare_npz_host_f32_v1`` as shipped
    (jittor_hybridsplat/ops/native/rasterizer/flashgs_prepare.cpp, built with
    the reference's Release flags by oracle/build_ref.py into
    ``oracle/_ref/libref_prepare.so``; single-threaded), both groups.
``cameras.opencv``
    ``load_camera_records`` (camera.py:142-220) at ratio 0.25.
``cameras.flashgs``
    ``load_flashgs_camera_records`` (camera.py:223-293).
``prepare_camera``
    a numpy float32 restatement of ``prepare_camera`` (camera.py:319-360)
    with ``focal_to_fov``, ``world_to_view`` and ``projection_matrix``
    (camera.py:19-61) and the camera centre -R^T T, for all 20 views.

``python oracle/cpu_stages.py [--reference PATH] [--runs 7]`` times every
stage, importing the reference's Python modules from its checkout (``--reference``,
else ``$HYBRIDSPLAT_REFERENCE_ROOT``, else ``../reference`` beside the
repository), checks the loaded contract and cameras against the generated
ones, and writes ``cpu_stages_config0.json`` beside this file. Where the
reference's Python is absent (a GPU host), ``host_stages()`` times the
stages that need only numpy and the prebuilt ``oracle/_ref`` library.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import platform
import statistics
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
REPO_DIR = ORACLE_DIR.parent
RESULTS = ORACLE_DIR / "cpu_stages_config0.json"
REF_PREPARE = ORACLE_DIR / "_ref" / "libref_prepare.so"

VIEWS = 20
WIDTH, HEIGHT, FOCAL = 1292, 839, 1000.0
# The loaders quarter the stored resolution and focal length
# (camera.py:183-189 at ratio 0.25, camera.py:268-283).
STORED_SCALE = 4
NEAR, FAR = 0.2, 20.0
GROUPS = (("base", "sampler.pcd"), ("reflection", "sampler.ref"))


def _scenes():
    if str(REPO_DIR) not in sys.path:
        sys.path.insert(0, str(REPO_DIR))
    from hybridsplat_jittor_render_b200 import scenes

    return scenes


def host_info() -> dict:
    model = platform.processor() or ""
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                model = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return {"cpu": model, "logical_cores": os.cpu_count(), "cores_available": len(os.sched_getaffinity(0)),
            "threads_used": 1}


# --------------------------------------------------------------------------
# Config-0 dataset on disk
# --------------------------------------------------------------------------

def checkpoint_members(scene: dict, degree: int = 3) -> dict[str, np.ndarray]:
    """The 29 NPZ members of the strict checkpoint contract
    (checkpoint.py:64-140: per group 13 members, two backgrounds, epoch)."""
    members: dict[str, np.ndarray] = {"epoch": np.array(30000, dtype="<i8"),
                                      "sampler.bg_color": np.zeros(3, "<f4"),
                                      "sampler.ref_bg_color": np.zeros(3, "<f4")}
    for group, prefix in GROUPS:
        g = scene[group]
        n = g["xyz"].shape[0]
        rest = (degree + 1) ** 2 - 1
        members.update({
            f"{prefix}.active_sh_degree": np.array([degree], dtype="<i8"),
            f"{prefix}._xyz": g["xyz"],
            f"{prefix}._features_dc": g["features_dc"],
            f"{prefix}._features_rest": np.ascontiguousarray(g["features_rest"][:, :rest]),
            f"{prefix}._scaling": g["scaling"],
            f"{prefix}._rotation": g["rotation"],
            f"{prefix}._opacity": g["opacity"],
            f"{prefix}._specular": g["specular"],
            f"{prefix}._roughness": g["roughness"],
            f"{prefix}.max_radii2D": np.zeros(n, "<f4"),
            f"{prefix}.xyz_gradient_accum": np.zeros((n, 1), "<f4"),
            f"{prefix}.denom": np.zeros((n, 1), "<f4"),
            f"{prefix}.xyz_weight_accum": np.zeros((n, 1), "<f4"),
        })
    return members


def _matrix(kind: str, name: str, m: np.ndarray) -> str:
    rows, cols = m.shape
    data = ", ".join(repr(float(v)) for v in m.reshape(-1))
    return (f"{kind}_{name}: !!opencv-matrix\n   rows: {rows}\n   cols: {cols}\n   dt: d\n"
            f"   data: [ {data} ]\n")


def write_dataset(root: Path) -> dict:
    """Writes checkpoint.npz, intri.yml, extri.yml and cameras.json for the
    CPU plumbing workload under `root`; returns the scene and cameras."""
    scenes = _scenes()
    scene = scenes.make_scene("cpu_plumbing")
    np.savez_compressed(root / "checkpoint.npz", **checkpoint_members(scene))
    cams = [scenes.orbit_camera("cpu_plumbing", v) for v in range(VIEWS)]
    names = [f"{v:03d}" for v in range(VIEWS)]
    intri, extri, flashgs = ["%YAML:1.0\n---\n"], ["%YAML:1.0\n---\n"], []
    for v, (name, cam) in enumerate(zip(names, cams)):
        k = np.array([[FOCAL * STORED_SCALE, 0.0, WIDTH * STORED_SCALE / 2.0],
                      [0.0, FOCAL * STORED_SCALE, HEIGHT * STORED_SCALE / 2.0], [0.0, 0.0, 1.0]])
        intri.append(_matrix("K", name, k))
        intri.append(f"H_{name}: {HEIGHT * STORED_SCALE}\nW_{name}: {WIDTH * STORED_SCALE}\n")
        extri.append(_matrix("Rot", name, cam.R.astype(np.float64)))
        extri.append(_matrix("T", name, cam.T.astype(np.float64).reshape(3, 1)))
        flashgs.append({"id": v, "img_name": name, "width": WIDTH * STORED_SCALE, "height": HEIGHT * STORED_SCALE,
                        "position": [float(x) for x in cam.center],
                        "rotation": cam.R.T.astype(np.float64).tolist(),
                        "fx": FOCAL * STORED_SCALE, "fy": FOCAL * STORED_SCALE})
    (root / "intri.yml").write_text("".join(intri))
    (root / "extri.yml").write_text("".join(extri))
    (root / "cameras.json").write_text(json.dumps(flashgs))
    return {"scene": scene, "cameras": cams, "names": names}


# --------------------------------------------------------------------------
# Restatements (numpy float32)
# --------------------------------------------------------------------------

def activate(group: dict[str, np.ndarray]) -> dict[str, np.ndarray]:
    """checkpoint.py:438-461 in numpy float32: exp scaling, rotation over
    max(|q|, 1e-12), logistic opacity/specular/roughness."""
    f32 = np.float32
    q = group["rotation"]
    norm = np.sqrt((q * q).sum(axis=-1, keepdims=True, dtype=f32))
    one = f32(1.0)
    return {"scaling": np.exp(group["scaling"]), "rotation": q / np.maximum(norm, f32(1e-12)),
            "opacity": one / (one + np.exp(-group["opacity"])),
            "specular": one / (one + np.exp(-group["specular"])),
            "roughness": one / (one + np.exp(-group["roughness"]))}


def prepare_camera(height: int, width: int, K, R, T, near, far, focal_x: float, focal_y: float) -> dict:
    """camera.py:319-360 with camera.py:19-61 in numpy float32: the FoVs from
    the focal lengths, world_view = [R|T; 0 0 0 1]^T, the projection
    transposed, their product and the centre -R^T T."""
    f32 = np.float32
    fov_x = 2.0 * math.atan(float(width) / (2.0 * float(focal_x)))
    fov_y = 2.0 * math.atan(float(height) / (2.0 * float(focal_y)))
    near = np.asarray(near, f32).reshape(1)
    far = np.asarray(far, f32).reshape(1)
    tan_x, tan_y = math.tan(fov_x * 0.5), math.tan(fov_y * 0.5)
    top = f32(tan_y) * near
    right = f32(tan_x) * near
    bottom, left = -top, -right
    proj = np.zeros((4, 4), f32)
    proj[0, 0] = (f32(2.0) * near / (right - left))[0]
    proj[1, 1] = (f32(2.0) * near / (top - bottom))[0]
    proj[0, 2] = ((right + left) / (right - left))[0]
    proj[1, 2] = ((top + bottom) / (top - bottom))[0]
    proj[2, 2] = (far / (far - near))[0]
    proj[2, 3] = (-(far * near) / (far - near))[0]
    proj[3, 2] = 1.0
    world_view = np.eye(4, dtype=f32)
    world_view[:3, :3] = R
    world_view[:3, 3:4] = T
    world_view = np.ascontiguousarray(world_view.T)
    projection = np.ascontiguousarray(proj.T)
    return {"image_height": int(height), "image_width": int(width), "FoVx": fov_x, "FoVy": fov_y,
            "tanfovx": tan_x, "tanfovy": tan_y, "world_view_transform": world_view,
            "projection_matrix": projection, "full_proj_transform": world_view @ projection,
            "camera_center": -(R.T @ T).reshape(3)}


def _bind_prepare(path: Path):
    lib = ctypes.CDLL(str(path))
    fn = lib.hs_flashgs_prepare_npz_host_f32_v1
    fn.restype = ctypes.c_int32
    fn.argtypes = [ctypes.c_uint64] + [ctypes.c_void_p] * 11 + [ctypes.c_char_p, ctypes.c_uint64]
    return fn


def flashgs_prepare(fn, group: dict[str, np.ndarray]) -> dict[str, np.ndarray]:
    """One group through the shipped host activation (flashgs_prepare.cpp)."""
    n = group["xyz"].shape[0]
    ins = [np.ascontiguousarray(group[k], np.float32) for k in ("opacity", "scaling", "rotation", "specular",
                                                                  "roughness")]
    outs = {"opacity": np.empty((n, 1), np.float32), "scaling": np.empty((n, 2), np.float32),
            "rotation": np.empty((n, 4), np.float32), "covariance": np.empty((n, 6), np.float32),
            "specular": np.empty((n, 1), np.float32), "roughness": np.empty((n, 1), np.float32)}
    err = ctypes.create_string_buffer(256)
    status = fn(n, *[a.ctypes.data for a in ins], *[a.ctypes.data for a in outs.values()], err, len(err))
    if status != 0:
        raise RuntimeError(f"hs_flashgs_prepare_npz_host_f32_v1 failed ({status}): {err.value.decode()}")
    return outs


# --------------------------------------------------------------------------
# Timing
# --------------------------------------------------------------------------

def median_ms(fn, runs: int) -> dict:
    fn()  # warm: file cache, imports, first-touch allocations
    times = []
    for _ in range(runs):
        t0 = time.perf_counter()
        fn()
        times.append((time.perf_counter() - t0) * 1e3)
    return {"ms": round(statistics.median(times), 4), "min_ms": round(min(times), 4), "runs": runs}


def camera_inputs(cams) -> list[tuple]:
    f32 = np.float32
    out = []
    for cam in cams:
        k = np.array([[FOCAL, 0, WIDTH / 2.0], [0, FOCAL, HEIGHT / 2.0], [0, 0, 1]], f32)
        out.append((HEIGHT, WIDTH, k, cam.R.astype(f32), cam.T.astype(f32).reshape(3, 1),
                    np.array([NEAR], f32), np.array([FAR], f32), FOCAL, FOCAL))
    return out


def host_stages(runs: int = 7, prepare_library: Path = REF_PREPARE) -> dict:
    """The stages that need no reference Python: the numpy restatements and
    the shipped host activation from the prebuilt oracle/_ref library."""
    scenes = _scenes()
    scene = scenes.make_scene("cpu_plumbing")
    cams = [scenes.orbit_camera("cpu_plumbing", v) for v in range(VIEWS)]
    stages = {"activation": median_ms(lambda: [activate(scene[g]) for g, _ in GROUPS], runs)}
    if prepare_library.exists():
        fn = _bind_prepare(prepare_library)
        stages["flashgs_prepare_host"] = median_ms(lambda: [flashgs_prepare(fn, scene[g]) for g, _ in GROUPS], runs)
    inputs = camera_inputs(cams)
    stages["prepare_camera"] = median_ms(lambda: [prepare_camera(*args) for args in inputs], runs)
    return stages


def default_reference() -> Path:
    env = os.environ.get("HYBRIDSPLAT_REFERENCE_ROOT")
    return Path(env) if env else REPO_DIR.parent / "reference"


def measure(reference: Path, runs: int) -> dict:
    sys.path.insert(0, str(reference))
    from jittor_hybridsplat import camera as ref_camera  # noqa: E402
    from jittor_hybridsplat import checkpoint as ref_checkpoint  # noqa: E402

    with tempfile.TemporaryDirectory() as tmp:
        root = Path(tmp)
        data = write_dataset(root)
        path = root / "checkpoint.npz"
        contract = ref_checkpoint.validate_checkpoint_archive(path)
        assert (contract.base_points, contract.reflection_points, contract.sh_degree) == (10_000, 2_000, 3), contract
        records = ref_camera.load_camera_records(root, ratio=0.25, near=NEAR, far=FAR)
        flashgs = ref_camera.load_flashgs_camera_records(root)
        assert len(records) == len(flashgs) == VIEWS
        for rec, fg, cam in zip(records, flashgs, data["cameras"]):
            assert (rec.image_width, rec.image_height) == (fg.image_width, fg.image_height) == (WIDTH, HEIGHT)
            assert rec.K[0, 0] == rec.K[1, 1] == fg.focal_x == fg.focal_y == FOCAL
            assert np.array_equal(rec.R, cam.R) and np.array_equal(rec.T.reshape(3), cam.T)
            assert np.array_equal(fg.rotation, cam.R.T) and np.array_equal(fg.position, cam.center)
            prepared = prepare_camera(rec.image_height, rec.image_width, rec.K, rec.R, rec.T, rec.near, rec.far,
                                      focal_x=float(rec.K[0, 0]), focal_y=float(rec.K[1, 1]))
            np.testing.assert_allclose(prepared["full_proj_transform"], cam.full_proj(), rtol=1e-6, atol=1e-6)
        stages = {
            "checkpoint.infer": median_ms(lambda: ref_checkpoint.infer_checkpoint_contract(path), runs),
            "checkpoint.validate": median_ms(lambda: ref_checkpoint.validate_checkpoint_archive(path), runs),
            "cameras.opencv": median_ms(lambda: ref_camera.load_camera_records(root, ratio=0.25, near=NEAR,
                                                                               far=FAR), runs),
            "cameras.flashgs": median_ms(lambda: ref_camera.load_flashgs_camera_records(root), runs),
        }
        file_bytes = path.stat().st_size
    stages.update(host_stages(runs))
    total = stages["checkpoint.validate"]["ms"] + sum(
        stages[k]["ms"] for k in ("activation", "flashgs_prepare_host", "cameras.opencv", "cameras.flashgs",
                                  "prepare_camera") if k in stages)
    return {
        "workload": "cpu_plumbing: strict 29-member NPZ, 10000 base + 2000 reflective Gaussians, SH degree 3, "
                    "seed 0; 20 orbit views 1292x839 fx=fy=1000 (OpenCV YAML + FlashGS cameras.json)",
        "checkpoint_bytes": file_bytes, "host": host_info(), "stages": stages,
        "total_ms": round(total, 4),
        "total_note": "checkpoint.validate (which repeats checkpoint.infer) + activation + flashgs_prepare_host "
                      "+ both camera loaders + prepare_camera for 20 views",
        "command": "python oracle/cpu_stages.py --runs %d" % runs,
    }


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    parser.add_argument("--reference", type=Path, default=None)
    parser.add_argument("--runs", type=int, default=7)
    parser.add_argument("--out", type=Path, default=RESULTS)
    args = parser.parse_args()
    if args.runs < 5:
        parser.error("--runs must be at least 5")
    reference = args.reference or default_reference()
    if not (reference / "jittor_hybridsplat" / "checkpoint.py").exists():
        print(f"reference checkout not found at {reference}; nothing measured", file=sys.stderr)
        return 1
    result = measure(reference, args.runs)
    args.out.write_text(json.dumps(result, indent=1) + "\n")
    print(json.dumps(result, indent=1))
    return 0


if __name__ == "__main__":
    sys.exit(main())
