"""Context, workspace and error behaviour of the C ABI on a GPU.

Mirrors the reference semantics: pair-capacity growth with an overflow retry
counter (flashgs_backend.cu:415-500), stats structs checked by size and ABI
(c_api.cpp:625-632), grow-only workspaces that can be released and rebuilt,
deterministic repeated calls, and status codes for invalid arguments.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from helpers import FLASHGS_OUT, bits_equal, fixture_inputs, camera_args
from hybridsplat_jittor_render_b200 import NativeRasterizerError, NativeRendererContext, ops
from hybridsplat_jittor_render_b200 import native_runtime as nr

pytestmark = pytest.mark.gpu


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def render(ctx, data, group="base", capacity=1 << 16):
    inputs = fixture_inputs(data, "flashgs", group)
    return ops.flashgs_forward(*[dev(v) for v in inputs.values()], use_sh=group == "base",
                               initial_pair_capacity=capacity, context=ctx, **camera_args(data))


def test_overflow_growth_is_counted_and_exact(golden):
    data = golden("small")
    expected = int(data["flashgs_base_out_rendered"][0])
    with NativeRendererContext(0) as ctx:
        out = render(ctx, data, capacity=16)
        stats = ctx.flashgs_workspace_stats()
        assert stats["overflow_retry_count"] == 1
        assert stats["pair_capacity"] == max(expected + 1, 16 + 4)
        assert stats["last_num_rendered"] == expected and stats["forward_calls"] == 1
        for name, value in zip(FLASHGS_OUT, out):
            assert bits_equal(value.cpu().numpy(), data[f"flashgs_base_out_{name}"]), name
        render(ctx, data, capacity=16)
        assert ctx.flashgs_workspace_stats()["overflow_retry_count"] == 1  # capacity persists


def test_repeated_calls_and_view_changes_are_deterministic(golden):
    small, ragged = golden("small"), golden("ragged")
    with NativeRendererContext(0) as ctx:
        first = [t.cpu().numpy() for t in render(ctx, small)]
        render(ctx, ragged, group="reflection")  # different size and pair count in between
        again = [t.cpu().numpy() for t in render(ctx, small)]
    for a, b in zip(first, again):
        assert bits_equal(a, b)


def test_release_workspace_then_render(golden):
    data = golden("background")
    with NativeRendererContext(0) as ctx:
        render(ctx, data)
        before = ctx.flashgs_workspace_stats()
        assert before["initialized"] == 1 and before["current_bytes"] > 0
        ctx.release_workspace()
        after = ctx.flashgs_workspace_stats()
        assert after["initialized"] == 0 and after["current_bytes"] == 0
        out = render(ctx, data)
        assert bits_equal(out.color.cpu().numpy(), data["flashgs_base_out_color"])


def test_stats_abi_mismatch_and_debug_capacity(golden):
    data = golden("small")
    with NativeRendererContext(0) as ctx:
        render(ctx, data)
        stats = nr.FlashgsWorkspaceStatsV1()
        stats.struct_size = 8
        stats.abi_version = 2
        err = nr.error_buffer()
        assert ctx.library.hs_flashgs_workspace_stats_v1(ctx.handle, ctypes.byref(stats), err, len(err)) == 2
        buf = np.zeros(8, np.float32)
        status = ctx.library.hs_flashgs_debug_copy_v1(ctx.handle, 1, 1, 1, *([buf.ctypes.data] * 11), err,
                                                      len(err))
        assert status == 4 and b"FlashGS debug copy" in err.value
        assert ctx.math_workspace_stats()["handles_ready"] == 1
        assert ctx.optix_workspace_stats()["scene_ready"] == 0


def test_prefiltered_violation_is_reported_not_trapped(golden):
    data = golden("culled")  # every Gaussian is behind the camera
    inputs = fixture_inputs(data, "standard", "base")
    w, h = (int(v) for v in data["camera_size"])
    with NativeRendererContext(0) as ctx:
        with pytest.raises(NativeRasterizerError) as info:
            ops.rasterize_forward(*[dev(v) for v in inputs.values()], width=w, height=h, scale_modifier=1.0,
                                  tan_fovx=0.5, tan_fovy=0.5, prefiltered=True, context=ctx)
        assert info.value.status == 4
        # the context stays usable
        out = ops.rasterize_forward(*[dev(v) for v in inputs.values()], width=w, height=h, scale_modifier=1.0,
                                    tan_fovx=0.5, tan_fovy=0.5, context=ctx)
        torch.cuda.synchronize()
        assert int(out.rendered.item()) == 0


def test_trace_scene_build_checks_arguments_like_the_reference():
    """hs_optix_build_scene_v1 rejects null buffers (status 1) and zero sizes
    or a zero signature (status 3) with the reference's texts
    (optix_backend.cpp:375-400); release without a scene is fine."""
    with NativeRendererContext(0) as ctx:
        err = nr.error_buffer()
        status = ctx.library.hs_optix_build_scene_v1(ctx.handle, None, 0, None, 0, 0, 0, None, err, len(err))
        assert status == 1 and b"null buffer" in err.value
        v = torch.zeros((4, 3), device="cuda")
        t = torch.tensor([[0, 1, 2]], dtype=torch.int32, device="cuda")
        st = torch.zeros(1, dtype=torch.int32, device="cuda")
        status = ctx.library.hs_optix_build_scene_v1(ctx.handle, v.data_ptr(), 4, t.data_ptr(), 1, 0, 0,
                                                     st.data_ptr(), err, len(err))
        assert status == 3 and b"dimensions or scalars" in err.value
        ctx.release_optix_scene()
