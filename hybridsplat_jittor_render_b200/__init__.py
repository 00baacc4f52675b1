"""B200-native (sm_100a) HybridSplat forward renderer.

A drop-in replacement for the reference's native library
``libhybridsplat_rasterizer.so`` (C ABI version 2): deterministic FlashGS and
standard five-channel 2DGS forward passes, reflection-ray generation and the
two-branch fusion, written as CUDA kernels for Blackwell. The Python modules
here bind that C ABI (``native_runtime``), expose tensor-level operators
with the reference's names (``ops``) and generate the synthetic scenes used
by the tests and benchmarks (``scenes``).
"""

from .native_runtime import (
    HS_RASTERIZER_ABI_VERSION,
    LIBRARY_PATH,
    NativeRasterizerError,
    NativeRendererContext,
    bind_library,
    load_native_library,
)

__all__ = [
    "HS_RASTERIZER_ABI_VERSION",
    "LIBRARY_PATH",
    "NativeRasterizerError",
    "NativeRendererContext",
    "bind_library",
    "load_native_library",
]
