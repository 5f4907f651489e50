"""opac1ty_b200 -- B200-native (sm_100a) fused 2-bit codebook dequant-matmul for opacc1ty.

Drop-in for opacc1ty's fused dequant path: the .bf2 layer layout, the quantize / benchmark
entry points, and a CUDA kernel manager in place of the Metal one.  The compute runs in
``libopc_b200.so`` (C ABI in include/opc_b200.h); there is no CPU fallback.
"""

__version__ = "0.1.0"

from .layer import DeviceLayer, prepare_layer, dequantize, gemv  # noqa: E402,F401

__all__ = ["DeviceLayer", "prepare_layer", "dequantize", "gemv", "__version__"]
