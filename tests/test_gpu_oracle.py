"""CUDA library vs the CPU oracle on the small fixture scenes.

Same statistical agreement as the oracle-vs-reference test (the oracle has
no bit-identical counterpart of the GPU's approximate instructions), run
through the C ABI on the GPU.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from cases import CASES
from helpers import FLASHGS_OUT, camera_args, fixture_inputs
from hybridsplat_jittor_render_b200 import NativeRendererContext, ops
from oracle import oracle
from test_oracle_golden import AGREEMENT, close_fraction

pytestmark = pytest.mark.gpu


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("case", [c.name for c in CASES])
def test_cuda_flashgs_agrees_with_oracle(golden, case):
    data = golden(case)
    inputs = fixture_inputs(data, "flashgs", "base")
    with NativeRendererContext(0) as ctx:
        out = ops.flashgs_forward(*[dev(v) for v in inputs.values()], use_sh=True, context=ctx,
                                  **camera_args(data))
        torch.cuda.synchronize()
    cpu = oracle.flashgs_forward(inputs, use_sh=True, **camera_args(data))
    assert int(out.rendered.item()) == cpu["rendered"]
    for name, value in zip(FLASHGS_OUT, out):
        assert close_fraction(value.cpu().numpy(), cpu[name]) >= AGREEMENT, name


@pytest.mark.parametrize("case", [c.name for c in CASES])
def test_cuda_standard_agrees_with_oracle(golden, case):
    data = golden(case)
    inputs = fixture_inputs(data, "standard", "base")
    w, h = (int(v) for v in data["camera_size"])
    with NativeRendererContext(0) as ctx:
        out = ops.rasterize_forward(*[dev(v) for v in inputs.values()], width=w, height=h, scale_modifier=1.0,
                                    tan_fovx=0.5, tan_fovy=0.5, context=ctx)
        torch.cuda.synchronize()
    cpu = oracle.standard_forward(inputs, width=w, height=h)
    assert int(out.rendered.item()) == cpu["rendered"]
    assert np.array_equal(out.radii.cpu().numpy(), cpu["radii"])
    assert close_fraction(out.color.cpu().numpy(), cpu["color"]) >= AGREEMENT
    assert close_fraction(out.auxiliary.cpu().numpy(), cpu["auxiliary"]) >= AGREEMENT
