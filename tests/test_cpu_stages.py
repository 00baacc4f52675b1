"""The CPU-stage baseline helpers (oracle/cpu_stages.py) on the CPU plumbing
workload: the checkpoint members follow the strict contract's schema
(jittor_hybridsplat/checkpoint.py:64-140), the numpy restatements of the
activations and of prepare_camera agree with the shipped host activation
and with the library's camera matrices, and the committed measurement
carries every stage with at least five runs."""

from __future__ import annotations

import json

import numpy as np
import pytest

from conftest import REF_PREPARE
from hybridsplat_jittor_render_b200 import scenes
from oracle import cpu_stages

STAGES = ("checkpoint.infer", "checkpoint.validate", "activation", "flashgs_prepare_host", "cameras.opencv",
          "cameras.flashgs", "prepare_camera")


@pytest.fixture(scope="module")
def scene():
    return scenes.make_scene("cpu_plumbing")


def test_checkpoint_members_follow_the_contract(scene):
    members = cpu_stages.checkpoint_members(scene)
    assert len(members) == 29
    assert members["epoch"].shape == () and members["epoch"].dtype.str == "<i8"
    for prefix, n in (("sampler.pcd", 10_000), ("sampler.ref", 2_000)):
        assert members[f"{prefix}.active_sh_degree"].tolist() == [3]
        assert members[f"{prefix}._xyz"].shape == (n, 3)
        assert members[f"{prefix}._features_dc"].shape == (n, 1, 3)
        assert members[f"{prefix}._features_rest"].shape == (n, 15, 3)
        assert members[f"{prefix}.max_radii2D"].shape == (n,)
        for key in ("_opacity", "_specular", "_roughness", "xyz_gradient_accum", "denom", "xyz_weight_accum"):
            assert members[f"{prefix}.{key}"].shape == (n, 1)
    for key, value in members.items():
        if key.endswith("active_sh_degree") or key == "epoch":
            continue
        assert value.dtype.str == "<f4" and value.flags.c_contiguous and np.isfinite(value).all(), key


def test_dataset_files(tmp_path):
    cpu_stages.write_dataset(tmp_path)
    with np.load(tmp_path / "checkpoint.npz") as archive:
        assert len(archive.files) == 29
    cams = json.loads((tmp_path / "cameras.json").read_text())
    assert len(cams) == cpu_stages.VIEWS
    assert {c["width"] // 4 for c in cams} == {1292} and {c["height"] // 4 for c in cams} == {839}
    assert (tmp_path / "intri.yml").read_text().count("!!opencv-matrix") == cpu_stages.VIEWS
    assert (tmp_path / "extri.yml").read_text().count("!!opencv-matrix") == 2 * cpu_stages.VIEWS


def test_prepare_camera_restatement_matches_the_library_cameras():
    cams = [scenes.orbit_camera("cpu_plumbing", v) for v in range(cpu_stages.VIEWS)]
    for cam, args in zip(cams, cpu_stages.camera_inputs(cams)):
        out = cpu_stages.prepare_camera(*args)
        assert np.array_equal(out["world_view_transform"], cam.world_view())
        np.testing.assert_allclose(out["full_proj_transform"], cam.full_proj(), rtol=1e-6, atol=1e-7)
        np.testing.assert_allclose(out["camera_center"], scenes.standard_camera_center(cam), rtol=0, atol=1e-6)
        assert out["tanfovx"] == pytest.approx(cam.tan_fovx, rel=1e-12)


def test_activation_restatement_against_the_shipped_host_activation(scene):
    if not REF_PREPARE.exists():
        pytest.skip("reference host build absent")
    fn = cpu_stages._bind_prepare(REF_PREPARE)
    for group in ("base", "reflection"):
        ours = cpu_stages.activate(scene[group])
        shipped = cpu_stages.flashgs_prepare(fn, scene[group])
        for key in ("opacity", "scaling", "rotation", "specular", "roughness"):
            np.testing.assert_allclose(ours[key], shipped[key], rtol=2e-6, atol=1e-7, err_msg=key)


def test_host_stages_and_committed_measurement():
    live = cpu_stages.host_stages(5)
    assert {"activation", "prepare_camera"} <= set(live)
    assert all(v["ms"] > 0 and v["runs"] == 5 for v in live.values())
    committed = json.loads(cpu_stages.RESULTS.read_text())
    assert set(committed["stages"]) == set(STAGES)
    assert all(v["runs"] >= 5 for v in committed["stages"].values())
    assert committed["host"]["threads_used"] == 1 and committed["host"]["logical_cores"] >= 1
