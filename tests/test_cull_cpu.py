"""The standard backend's culling never drops a live quadrant.

The library emits, per Gaussian, only the tiles of its reference rectangle
whose widened x-range meets the row spans of its culling ellipse or disc, and
marks the 8x8 quadrants to evaluate. The oracle restates that geometry in C
(correctly rounded in place of the GPU's approximate square roots, whose
error is far inside the 0.03% + one-pixel widening) and checks it against the
reference's per-pixel alpha test: every quadrant holding a pixel that reaches
alpha >= 1/255 must be emitted with its bit set. Scenes follow the benchmark
distributions (the benchmark scene, the 6M scene and the inflated-scale 4K
stress scene), scaled down, from orbit and off-axis cameras.
"""

from __future__ import annotations

import numpy as np
import pytest

from hybridsplat_jittor_render_b200 import scenes
from oracle import oracle


@pytest.mark.parametrize("name,scale,camera", [
    ("standard_1m", 0.03, "orbit0"), ("standard_1m", 0.03, "generic2"),
    ("large_6m", 0.005, "orbit5"), ("stress_4k", 0.003, "generic1"),
])
def test_culling_keeps_every_live_quadrant(name, scale, camera):
    scene = scenes.make_scene(name, scale=scale)
    cam = scenes.orbit_camera(name, int(camera[5:])) if camera.startswith("orbit") else \
        scenes.generic_camera(name, int(camera[7:]))
    for group in ("base", "reflection"):
        g = scene[group]
        inputs = {"means3d": g["xyz"], "opacities": oracle.precise_sigmoid(g["opacity"]),
                  "scales": oracle.precise_exp(g["scaling"]), "rotations": oracle.precise_normalize4(g["rotation"]),
                  "viewmatrix": cam.world_view(), "projmatrix": cam.full_proj()}
        r = oracle.standard_cull_check(inputs, width=cam.width, height=cam.height)
        assert r["live_quadrants"] > 1000, r
        assert r["missed"] == 0, r
        # the culling removes part of the reference rectangles (the point of it)
        assert r["emitted_tiles"] < r["rect_tiles"], r
