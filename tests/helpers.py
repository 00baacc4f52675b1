"""Helpers shared by the tests: fixture unpacking and comparison metrics."""

from __future__ import annotations

import numpy as np

FLASHGS_OUT = ("color", "other", "depth", "alpha", "normal", "median_depth", "distortion")
FLASHGS_INPUTS = ("positions", "shs", "colors", "opacities", "covariance", "scales", "rotations", "specular",
                  "roughness")
STANDARD_INPUTS = ("background", "means3d", "colors", "opacities", "scales", "rotations", "viewmatrix",
                   "projmatrix", "camera_position")
DEBUG_FIELDS = ("points_xy", "rgb", "other_features", "conic_opacity", "normal_opacity", "Tu", "Tv", "Tw",
                "sorted_keys", "sorted_values", "tile_ranges")
# Tolerance of the standard backend (north star): per channel max-abs and mean-abs.
STANDARD_MAX_ABS = 1e-5
STANDARD_MEAN_ABS = 1e-7


def fixture_inputs(data: dict, backend: str, group: str) -> dict:
    names = FLASHGS_INPUTS if backend == "flashgs" else STANDARD_INPUTS
    return {k: data[f"{backend}_{group}_in_{k}"] for k in names}


def camera_args(data: dict) -> dict:
    w, h = (int(v) for v in data["camera_size"])
    fx, fy = (float(v) for v in data["camera_focal"])
    return dict(width=w, height=h, camera_position=[float(v) for v in data["camera_center"]],
                camera_rotation=[float(v) for v in data["camera_flashgs_rotation9"]], focal_x=fx, focal_y=fy,
                background=tuple(float(v) for v in data["background"]))


def bits_equal(a, b) -> bool:
    a, b = np.ascontiguousarray(a), np.ascontiguousarray(b)
    if a.shape != b.shape:
        return False
    if a.dtype.kind == "f":
        return bool(np.array_equal(a.view(np.uint32 if a.itemsize == 4 else np.uint64),
                                   b.view(np.uint32 if b.itemsize == 4 else np.uint64)))
    return bool(np.array_equal(a, b))


def channel_errors(a: np.ndarray, b: np.ndarray) -> list[tuple[float, float]]:
    """(max-abs, mean-abs) per leading channel; NaN/Inf count as infinite error."""
    out = []
    for ca, cb in zip(a.reshape(a.shape[0], -1), b.reshape(b.shape[0], -1)):
        d = np.abs(ca.astype(np.float64) - cb.astype(np.float64))
        d[~np.isfinite(d)] = np.inf
        out.append((float(d.max()) if d.size else 0.0, float(d.mean()) if d.size else 0.0))
    return out


def within_standard_tolerance(a: np.ndarray, b: np.ndarray) -> bool:
    return all(mx <= STANDARD_MAX_ABS and mn <= STANDARD_MEAN_ABS for mx, mn in channel_errors(a, b)) and \
        bool(np.isfinite(a).all())
