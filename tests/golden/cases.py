"""Fixture cases shared by the golden-vector generator and the tests.

Each case is a small seeded scene plus camera, sized so the CPU oracle
finishes in well under a second. The generator stores the inputs together
with the reference outputs (tests/golden/*.npz).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from hybridsplat_jittor_render_b200 import scenes


@dataclass(frozen=True)
class Case:
    name: str
    base: int
    reflection: int
    width: int
    height: int
    focal: float
    camera_seed: int = 0
    background: tuple[float, float, float] = (0.0, 0.0, 0.0)
    look_away: bool = False
    xyz_sigma: float = 1.0


CASES = [
    # config-0 distributions at a small resolution; generic (rolled) camera
    Case("small", 2000, 400, 96, 72, 90.0),
    # ragged image: partial tiles on both edges, pixels outside the image
    Case("ragged", 600, 120, 37, 29, 35.0, camera_seed=1),
    # non-zero background: encode() on empty tiles, T*bg on covered pixels
    Case("background", 300, 60, 64, 48, 60.0, camera_seed=2, background=(0.3, 0.7, 1.2)),
    # every Gaussian behind the camera: empty frame
    Case("culled", 200, 40, 48, 32, 45.0, look_away=True),
    # no Gaussians at all
    Case("empty", 0, 0, 40, 24, 40.0),
]


def camera_for(case: Case) -> scenes.Camera:
    spec = scenes.SceneSpec(case.name, scenes.GroupSpec(1), scenes.GroupSpec(1), case.width, case.height,
                            case.focal)
    cam = scenes.generic_camera(spec, case.camera_seed)
    if case.look_away:
        cam = scenes.look_at_camera(spec, cam.center, 2.0 * cam.center, roll_deg=30.0)
    return cam


def raw_groups(case: Case) -> dict[str, dict[str, np.ndarray]]:
    rng = np.random.default_rng(7)
    base = scenes.make_group(rng, scenes.GroupSpec(case.base, xyz_sigma=case.xyz_sigma))
    refl = scenes.make_group(rng, scenes.GroupSpec(case.reflection, xyz_sigma=case.xyz_sigma))
    return {"base": base, "reflection": refl}
