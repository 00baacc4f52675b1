"""Seeded synthetic HybridSplat scenes and orbit cameras.

The benchmark scene of the reference (Ref-Real "sedan", trained NPZ) is not
available, so scenes are drawn from the distributions of the benchmark
configurations: per Gaussian group, in the NPZ member order of the reference
checkpoint contract (jittor_hybridsplat/checkpoint.py:64-140) -- xyz, SH DC,
SH rest, log-scale, quaternion, opacity logit, specular logit, roughness
logit -- from one ``numpy.random.default_rng(seed)``, base group first.

Cameras follow the reference conventions:
  * OpenCV extrinsics: R rows are (right, down, forward), T = -R C
    (camera.py:142-220); the standard backend uses world_view = [R|T]^T and
    full_proj = world_view @ projection^T (camera.py:31-61, 319-360).
  * FlashGS: position C and rotation = R^T as 9 row-major floats, read as
    glm::mat3 columns by the backend (flashgs_backend.cu:424-430).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

SH_COEFFICIENTS = 16


@dataclass(frozen=True)
class GroupSpec:
    count: int
    xyz_sigma: float = 1.5
    log_scale: tuple[float, float] = (-4.0, 0.5)
    opacity_logit: tuple[float, float] = (0.0, 1.5)
    specular_logit: tuple[float, float] = (-1.0, 1.0)
    roughness_logit: tuple[float, float] = (0.0, 1.0)


@dataclass(frozen=True)
class SceneSpec:
    name: str
    base: GroupSpec
    reflection: GroupSpec
    width: int
    height: int
    focal: float
    views: int = 1
    radius: float = 4.0
    elevation_deg: float = 15.0
    azimuth_step_deg: float = 18.0
    seed: int = 0


# Benchmark configurations (sizes of the reference's benchmark matrix).
SCENES: dict[str, SceneSpec] = {
    "cpu_plumbing": SceneSpec("cpu_plumbing", GroupSpec(10_000, xyz_sigma=1.0), GroupSpec(2_000, xyz_sigma=1.0),
                              1292, 839, 1000.0, views=20),
    "standard_1m": SceneSpec("standard_1m", GroupSpec(1_000_000), GroupSpec(200_000), 1292, 839, 1000.0),
    "flashgs_1m": SceneSpec("flashgs_1m", GroupSpec(1_000_000), GroupSpec(200_000), 1292, 839, 1000.0, views=20),
    "large_6m": SceneSpec("large_6m", GroupSpec(6_000_000, log_scale=(-4.5, 0.6)),
                          GroupSpec(1_000_000, log_scale=(-4.5, 0.6)), 1920, 1080, 1400.0, views=160),
    "stress_4k": SceneSpec("stress_4k", GroupSpec(3_000_000, log_scale=(-3.0, 0.5), opacity_logit=(1.0, 1.0)),
                           GroupSpec(500_000, log_scale=(-3.0, 0.5), opacity_logit=(1.0, 1.0)),
                           3840, 2160, 2800.0),
}


def make_group(rng: np.random.Generator, spec: GroupSpec) -> dict[str, np.ndarray]:
    """Raw (pre-activation) arrays of one Gaussian group, float32."""
    n = spec.count
    f32 = np.float32
    group = {
        "xyz": rng.normal(0.0, spec.xyz_sigma, (n, 3)).astype(f32),
        "features_dc": rng.normal(0.0, 0.5, (n, 1, 3)).astype(f32),
        "features_rest": rng.normal(0.0, 0.05, (n, SH_COEFFICIENTS - 1, 3)).astype(f32),
        "scaling": rng.normal(spec.log_scale[0], spec.log_scale[1], (n, 2)).astype(f32),
        "rotation": rng.normal(0.0, 1.0, (n, 4)).astype(f32),
        "opacity": rng.normal(spec.opacity_logit[0], spec.opacity_logit[1], (n, 1)).astype(f32),
        "specular": rng.normal(spec.specular_logit[0], spec.specular_logit[1], (n, 1)).astype(f32),
        "roughness": rng.normal(spec.roughness_logit[0], spec.roughness_logit[1], (n, 1)).astype(f32),
    }
    return group


# Rows per independently seeded chunk of a scene array (make_scene).
_CHUNK_ROWS = 1 << 18


def _normal_f32(seed: np.random.SeedSequence, shape: tuple[int, ...], mean: float, sigma: float,
                pool) -> np.ndarray:
    """float32 N(mean, sigma) array of `shape`, drawn in fixed chunks of rows
    from child seeds of `seed` (so the values do not depend on the thread
    count) on the threads of `pool`."""
    out = np.empty(shape, np.float32)
    rows = shape[0]
    starts = list(range(0, rows, _CHUNK_ROWS))
    children = seed.spawn(len(starts))

    def fill(k: int) -> None:
        a, b = starts[k], min(rows, starts[k] + _CHUNK_ROWS)
        chunk = out[a:b]
        np.random.default_rng(children[k]).standard_normal(chunk.shape, dtype=np.float32, out=chunk)
        chunk *= np.float32(sigma)
        chunk += np.float32(mean)

    list(pool.map(fill, range(len(starts))))
    return out


def make_scene(spec: SceneSpec | str, *, scale: float = 1.0) -> dict[str, dict[str, np.ndarray]]:
    """Both groups of a scene; `scale` < 1 shrinks the Gaussian counts.

    Arrays are drawn in float32 from per-array, per-chunk child seeds of the
    scene seed (numpy SeedSequence), in the NPZ member order of make_group,
    on the host's cores: a 7M-Gaussian scene takes seconds, not minutes."""
    from concurrent.futures import ThreadPoolExecutor
    import os

    if isinstance(spec, str):
        spec = SCENES[spec]

    def scaled(g: GroupSpec) -> GroupSpec:
        return GroupSpec(max(1, int(round(g.count * scale))), g.xyz_sigma, g.log_scale, g.opacity_logit,
                         g.specular_logit, g.roughness_logit)

    root = np.random.SeedSequence(spec.seed)
    group_seeds = root.spawn(2)
    out = {}
    workers = max(1, min(16, len(os.sched_getaffinity(0))))
    with ThreadPoolExecutor(workers) as pool:
        for name, g, seed in (("base", scaled(spec.base), group_seeds[0]),
                              ("reflection", scaled(spec.reflection), group_seeds[1])):
            n = g.count
            fields = [("xyz", (n, 3), 0.0, g.xyz_sigma), ("features_dc", (n, 1, 3), 0.0, 0.5),
                      ("features_rest", (n, SH_COEFFICIENTS - 1, 3), 0.0, 0.05),
                      ("scaling", (n, 2), *g.log_scale), ("rotation", (n, 4), 0.0, 1.0),
                      ("opacity", (n, 1), *g.opacity_logit), ("specular", (n, 1), *g.specular_logit),
                      ("roughness", (n, 1), *g.roughness_logit)]
            seeds = seed.spawn(len(fields))
            out[name] = {key: _normal_f32(sd, shape, mean, sigma, pool)
                         for (key, shape, mean, sigma), sd in zip(fields, seeds)}
    return out


def sh_features(group: dict[str, np.ndarray]) -> np.ndarray:
    """[P, 16, 3] SH coefficients (DC first), the layout FlashGS reads as [P, 48]."""
    return np.ascontiguousarray(np.concatenate([group["features_dc"], group["features_rest"]], axis=1))


def sigmoid(x: np.ndarray) -> np.ndarray:
    return (1.0 / (1.0 + np.exp(-x.astype(np.float64)))).astype(np.float32)


@dataclass
class Camera:
    width: int
    height: int
    fx: float
    fy: float
    R: np.ndarray          # world -> camera rotation, rows (right, down, forward)
    T: np.ndarray          # [3]
    center: np.ndarray     # [3]
    znear: float = 0.2
    zfar: float = 20.0
    flashgs_znear: float = 0.01
    flashgs_zfar: float = 100.0
    extras: dict = field(default_factory=dict)

    @property
    def flashgs_rotation9(self) -> list[float]:
        return [float(v) for v in self.R.T.reshape(-1)]

    @property
    def flashgs_position(self) -> list[float]:
        return [float(v) for v in self.center]

    @property
    def tan_fovx(self) -> float:
        return math.tan(math.atan(self.width / (2.0 * self.fx)))

    @property
    def tan_fovy(self) -> float:
        return math.tan(math.atan(self.height / (2.0 * self.fy)))

    def world_view(self) -> np.ndarray:
        """[4,4] float32 storage read by the standard backend (= [R|T]^T)."""
        w = np.eye(4, dtype=np.float32)
        w[:3, :3] = self.R
        w[:3, 3] = self.T
        return np.ascontiguousarray(w.T)

    def projection(self) -> np.ndarray:
        tan_x, tan_y = self.tan_fovx, self.tan_fovy
        n, f = np.float32(self.znear), np.float32(self.zfar)
        top = np.float32(tan_y) * n
        right = np.float32(tan_x) * n
        p = np.zeros((4, 4), np.float32)
        p[0, 0] = 2.0 * n / (right + right)
        p[1, 1] = 2.0 * n / (top + top)
        p[2, 2] = f / (f - n)
        p[2, 3] = -(f * n) / (f - n)
        p[3, 2] = 1.0
        return p

    def full_proj(self) -> np.ndarray:
        """world_view @ projection^T (row-vector convention, float32)."""
        return np.ascontiguousarray(self.world_view() @ self.projection().T)


def orbit_camera(spec: SceneSpec | str, view: int) -> Camera:
    if isinstance(spec, str):
        spec = SCENES[spec]
    az = math.radians(spec.azimuth_step_deg * view)
    el = math.radians(spec.elevation_deg)
    center = np.array([spec.radius * math.cos(el) * math.cos(az),
                       spec.radius * math.cos(el) * math.sin(az),
                       spec.radius * math.sin(el)], np.float64)
    forward = -center / np.linalg.norm(center)
    up = np.array([0.0, 0.0, 1.0])
    right = np.cross(forward, up)
    right /= np.linalg.norm(right)
    down = np.cross(forward, right)
    R = np.stack([right, down, forward]).astype(np.float32)
    C = center.astype(np.float32)
    T = (-(R.astype(np.float64) @ C.astype(np.float64))).astype(np.float32)
    return Camera(spec.width, spec.height, spec.focal, spec.focal, R, T, C)


def look_at_camera(spec: SceneSpec | str, center, target=(0.0, 0.0, 0.0), roll_deg: float = 0.0) -> Camera:
    """Camera at `center` looking at `target`, rolled about its forward axis."""
    if isinstance(spec, str):
        spec = SCENES[spec]
    center = np.asarray(center, np.float64)
    forward = np.asarray(target, np.float64) - center
    forward /= np.linalg.norm(forward)
    up = np.array([0.0, 0.0, 1.0])
    right = np.cross(forward, up)
    right /= np.linalg.norm(right)
    down = np.cross(forward, right)
    roll = math.radians(roll_deg)
    right, down = (math.cos(roll) * right + math.sin(roll) * down,
                   -math.sin(roll) * right + math.cos(roll) * down)
    R = np.stack([right, down, forward]).astype(np.float32)
    C = center.astype(np.float32)
    T = (-(R.astype(np.float64) @ C.astype(np.float64))).astype(np.float32)
    return Camera(spec.width, spec.height, spec.focal, spec.focal, R, T, C)


def generic_camera(spec: SceneSpec | str, seed: int = 0) -> Camera:
    """Off-axis, rolled camera on the orbit sphere. Its rotation has no zero
    entries, so every product of the projection contributes (orbit cameras
    keep the right vector horizontal, which zeroes some matrix entries)."""
    if isinstance(spec, str):
        spec = SCENES[spec]
    rng = np.random.default_rng(1000 + seed)
    az = rng.uniform(0, 2 * math.pi)
    el = rng.uniform(math.radians(5), math.radians(40))
    c = spec.radius * np.array([math.cos(el) * math.cos(az), math.cos(el) * math.sin(az), math.sin(el)])
    target = rng.normal(0.0, 0.3, 3)
    return look_at_camera(spec, c, target, roll_deg=float(rng.uniform(10, 80)))


def standard_camera_center(camera: Camera) -> np.ndarray:
    """-R^T T in float32 (the quantity precise_camera_center produces)."""
    return (-(camera.R.T.astype(np.float32) @ camera.T.astype(np.float32))).astype(np.float32)
