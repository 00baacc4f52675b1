"""CPU restatement of the sessions' raw-map postprocess (numpy, float32).

TEST INFRASTRUCTURE ONLY: the parity tests compare the CUDA library's fused
postprocess (hs_b200_standard_postprocess_f32_v1,
hs_b200_flashgs_postprocess_f32_v1) with this restatement; the product never
imports it.

Restates, operation by operation in IEEE float32 (every product, sum, quotient
and square root rounded on its own):
  standard  postprocess_raster       math.py:426-463
            depth_to_normal           math.py:351-423 (from its world-space rays)
            _nan_to_num_like_pytorch  math.py:331-336
            safe_normalize            math.py:15-18
            precise_depth_divide      ops/jittor/precise_depth_divide_op.cc
  FlashGS   _flashgs_postprocess      renderer.py:176-202
The pixel rays come from the two TF32 GEMMs of depth_to_normal, which have no
CPU counterpart; callers pass the rays the GPU computed. The reference runs the
3-term normal rotation, the cross product and the squared norm as framework
kernels whose fused multiply-adds are its code generator's choice; here each
is a plain sequence of rounded operations, in the order the expressions are
written.
"""

from __future__ import annotations

import numpy as np

F32 = np.float32
FLT_MAX_NEG = np.float32(-3.4028234663852886e38)


def nan_to_num_session(v: np.ndarray) -> np.ndarray:
    """NaN and +inf -> 0, -inf -> -FLT_MAX (math.py:331-336)."""
    v = np.asarray(v, F32)
    out = np.where(np.isnan(v), F32(0), v)
    out = np.where(np.isposinf(out), F32(0), out)
    return np.where(np.isneginf(out), FLT_MAX_NEG, out).astype(F32)


def depth_divide(numerator: np.ndarray, denominator: np.ndarray) -> np.ndarray:
    """Correctly rounded quotient, NaN/+inf -> 0, -inf -> -FLT_MAX."""
    with np.errstate(all="ignore"):
        q = np.divide(np.asarray(numerator, F32), np.asarray(denominator, F32), dtype=F32)
    return nan_to_num_session(q)


def rotate_rows(n: np.ndarray, b: np.ndarray) -> np.ndarray:
    """n[...,3] @ b[3,3] as (n0*b0j + n1*b1j) + n2*b2j."""
    n = np.asarray(n, F32)
    b = np.asarray(b, F32)
    cols = [((n[..., 0] * b[0, j]).astype(F32) + (n[..., 1] * b[1, j]).astype(F32)).astype(F32)
            + (n[..., 2] * b[2, j]).astype(F32) for j in range(3)]
    return np.stack([c.astype(F32) for c in cols], -1)


def standard_postprocess(color: np.ndarray, aux: np.ndarray, rays: np.ndarray, origin: np.ndarray,
                         normal_rotation: np.ndarray, depth_ratio: float = 0.0) -> dict[str, np.ndarray]:
    """Maps of postprocess_raster from color[5,H,W], aux[7,H,W] and the view's
    world-space pixel rays [H*W,3]; each map [1,H*W,C]."""
    color = np.asarray(color, F32)
    aux = np.asarray(aux, F32)
    _, h, w = color.shape
    keep, ratio = F32(1.0 - float(depth_ratio)), F32(depth_ratio)
    alpha = aux[1]
    with np.errstate(all="ignore"):
        normal = rotate_rows(np.moveaxis(aux[2:5], 0, -1), normal_rotation)
        expected = depth_divide(aux[0], alpha)
        median = nan_to_num_session(aux[5])
        depth = ((expected * keep).astype(F32) + (median * ratio).astype(F32)).astype(F32)
        xyz = ((depth.reshape(-1, 1) * np.asarray(rays, F32)).astype(F32) + np.asarray(origin, F32)).astype(F32)
        xyz = xyz.reshape(h, w, 3)
        dx = (xyz[2:, 1:-1] - xyz[:-2, 1:-1]).astype(F32)
        dy = (xyz[1:-1, 2:] - xyz[1:-1, :-2]).astype(F32)
        cross = np.stack([
            ((dx[..., 1] * dy[..., 2]).astype(F32) - (dx[..., 2] * dy[..., 1]).astype(F32)).astype(F32),
            ((dx[..., 2] * dy[..., 0]).astype(F32) - (dx[..., 0] * dy[..., 2]).astype(F32)).astype(F32),
            ((dx[..., 0] * dy[..., 1]).astype(F32) - (dx[..., 1] * dy[..., 0]).astype(F32)).astype(F32)], -1)
        sq = (cross * cross).astype(F32)
        norm = np.sqrt(((sq[..., 0] + sq[..., 1]).astype(F32) + sq[..., 2]).astype(F32)).astype(F32)
        norm = np.maximum(norm, F32(1e-12))
        inner = (cross / norm[..., None]).astype(F32)
        surface = np.zeros((h, w, 3), F32)
        surface[1:-1, 1:-1] = inner
        surface = (surface * alpha[..., None]).astype(F32)

    def flat(hwc: np.ndarray) -> np.ndarray:
        return np.ascontiguousarray(hwc.reshape(1, h * w, -1), F32)

    return {
        "rgb_map": flat(np.moveaxis(color[:3], 0, -1)),
        "acc_map": flat(alpha[..., None]),
        "dpt_map": flat(depth[..., None]),
        "norm_map": flat(normal),
        "surf_norm_map": flat(surface),
        "dist_map": flat(aux[6][..., None]),
        "spec_map": flat(color[3][..., None]),
        "rough_map": flat(color[4][..., None]),
    }


def flashgs_postprocess(color: np.ndarray, other: np.ndarray, depth: np.ndarray, alpha: np.ndarray,
                        normal: np.ndarray, normal_rotation: np.ndarray) -> dict[str, np.ndarray]:
    """Maps of _flashgs_postprocess from a FlashGS forward's planes."""
    color, other = np.asarray(color, F32), np.asarray(other, F32)
    alpha = np.asarray(alpha, F32).reshape(color.shape[1:])
    h, w = alpha.shape

    def flat(hwc: np.ndarray) -> np.ndarray:
        return np.ascontiguousarray(hwc.reshape(1, h * w, -1), F32)

    with np.errstate(all="ignore"):
        dpt = nan_to_num_session(depth_divide(np.asarray(depth, F32).reshape(h, w), alpha))
        rotated = rotate_rows(np.moveaxis(np.asarray(normal, F32), 0, -1), normal_rotation)
    return {
        "rgb_map": flat(np.moveaxis(color, 0, -1)),
        "acc_map": flat(alpha[..., None]),
        "dpt_map": flat(dpt[..., None]),
        "norm_map": flat(rotated),
        "surf_norm_map": np.zeros((1, h * w, 3), F32),
        "dist_map": np.zeros((1, h * w, 1), F32),
        "spec_map": flat(other[0][..., None]),
    }
