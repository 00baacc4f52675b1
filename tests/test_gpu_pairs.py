"""The packed FP32x2 arithmetic of the rasterisers (hs_b200_test_pair_ops_v1).

Each lane of the rasterisers evaluates two pixels with sm_100 pair
instructions; their outputs equal the reference's only if every component of
every packed helper rounds exactly as the scalar helper it mirrors. The
library's self-check compares the two bit for bit over all variants; the
inputs here mix random values of every magnitude with signed zeros,
subnormals, infinities, NaNs and values near overflow, in both lanes of a pair.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from hybridsplat_jittor_render_b200 import native_runtime as nr

pytestmark = pytest.mark.gpu

OPS = ["mul", "add", "sub", "fma", "mad0", "mad1", "msub0", "msub1", "nmad0", "nmad1",
       "dot2_0", "dot2_1", "dot2_2", "diff2_0", "diff2_1", "diff2_2"]

SPECIAL = np.array([0.0, -0.0, 1.0, -1.0, np.inf, -np.inf, np.nan, 1e-45, -1e-45, 1e-40, -3e-39, 1.17549435e-38,
                    3.4028235e38, -3.4028235e38, 1e38, 1e-38, 0.5, 3.0, 1.0000001, 0.99999994], dtype=np.float32)


def operands(n: int, seed: int) -> list[np.ndarray]:
    """Four operand arrays: values of every binade (subnormals included), a
    third of typical magnitude, 5% special values, and the first k*k entries of
    the first two arrays every pair of special values."""
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(4):
        mantissa = rng.uniform(-2.0, 2.0, n)
        exponent = rng.integers(-150, 128, n).astype(np.float64)
        with np.errstate(over="ignore"):
            v = (mantissa * np.exp2(exponent)).astype(np.float32)
        typical = rng.random(n) < 0.3
        v[typical] = rng.standard_normal(int(typical.sum())).astype(np.float32)
        special = rng.random(n) < 0.05
        v[special] = rng.choice(SPECIAL, int(special.sum()))
        out.append(v)
    k = len(SPECIAL)
    grid = np.stack(np.meshgrid(np.arange(k), np.arange(k)), -1).reshape(-1, 2)
    if n >= grid.shape[0]:
        for j in range(2):
            out[j][: grid.shape[0]] = SPECIAL[grid[:, j]]
    return out


def run(n: int, seed: int) -> dict[str, int]:
    lib = nr.load_native_library()
    a, b, c, d = (torch.from_numpy(x).cuda() for x in operands(n, seed))
    mismatches = torch.zeros(16, dtype=torch.int32, device="cuda")
    err = ctypes.create_string_buffer(256)
    status = lib.hs_b200_test_pair_ops_v1(a.data_ptr(), b.data_ptr(), c.data_ptr(), d.data_ptr(), n,
                                          mismatches.data_ptr(), err, len(err))
    assert status == 0, err.value
    torch.cuda.synchronize()
    return dict(zip(OPS, mismatches.cpu().tolist()))


@pytest.mark.parametrize("seed", [0, 1])
def test_packed_helpers_round_as_the_scalar_ones(seed):
    counts = run(1 << 22, seed)
    assert all(v == 0 for v in counts.values()), counts


def test_pair_check_reports_nothing_for_empty_input():
    assert run(1, 2) == dict.fromkeys(OPS, 0)
