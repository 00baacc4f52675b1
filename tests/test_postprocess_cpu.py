"""CPU checks of the postprocess restatement (oracle/postprocess.py).

The non-finite mapping of the sessions' depth divide and nan_to_num, the
border and alpha handling of the surface normals, and a plane's surface
normal from exact rays, on inputs small enough to reason about by hand.
"""

from __future__ import annotations

import numpy as np

from oracle import postprocess as restated


def test_non_finite_mapping():
    v = np.array([np.nan, np.inf, -np.inf, 1.5, -0.0], np.float32)
    out = restated.nan_to_num_session(v)
    assert out.tolist()[:4] == [0.0, 0.0, float(np.float32(-3.4028234663852886e38)), 1.5]
    assert np.signbit(out[4])
    q = restated.depth_divide(np.array([1, -1, 0, 3], np.float32), np.array([0, 0, 0, 2], np.float32))
    assert q.tolist() == [0.0, float(np.float32(-3.4028234663852886e38)), 0.0, 1.5]


def test_plane_surface_normals_and_borders():
    """A fronto-parallel plane at depth 2 seen through rays (x, y, 1): interior
    surface normals are +-z, scaled by alpha; the border is zero."""
    h, w = 5, 6
    ys, xs = np.mgrid[0:h, 0:w].astype(np.float32)
    rays = np.stack([xs, ys, np.ones_like(xs)], -1).reshape(-1, 3)
    color = np.zeros((5, h, w), np.float32)
    aux = np.zeros((7, h, w), np.float32)
    aux[1] = 0.5          # alpha
    aux[0] = 1.0          # alpha-weighted depth: expected depth 2
    aux[5] = np.nan       # median: mapped to 0
    maps = restated.standard_postprocess(color, aux, rays, np.zeros(3, np.float32), np.eye(3, dtype=np.float32))
    assert np.all(maps["dpt_map"] == 2.0)
    surf = maps["surf_norm_map"].reshape(h, w, 3)
    assert np.all(surf[0] == 0) and np.all(surf[-1] == 0) and np.all(surf[:, 0] == 0) and np.all(surf[:, -1] == 0)
    interior = surf[1:-1, 1:-1]
    assert np.allclose(np.abs(interior[..., 2]), 0.5) and np.all(interior[..., :2] == 0)
    # depth_ratio blends the (mapped) median in: 2 * 0.75 + 0 * 0.25
    blended = restated.standard_postprocess(color, aux, rays, np.zeros(3, np.float32), np.eye(3, dtype=np.float32),
                                            depth_ratio=0.25)
    assert np.all(blended["dpt_map"] == 1.5)
