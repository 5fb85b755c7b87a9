"""ferret_b200: B200-native quantized MoE W13 (gate+up) grouped GEMM.

The compute path is the in-tree CUDA library ``libferret_moe.so`` (sm_100a
tcgen05 / TMA kernels behind a C ABI, ``include/ferret_moe.h``); this package
binds it with ctypes and adds the torch-facing operators and the
expert-parallel layer.  Importing ``ferret_b200.ops`` fails loudly when the
library has not been built (``python -m ferret_b200.build``).
"""
__all__ = ["ops", "data", "build"]
__version__ = "0.1.0"
