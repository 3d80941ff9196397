"""B200-native (sm_100a) int4 KV-cache decode-attention path of svv232/gemma4metal.

The product is the shared library libturboquant_b200.so (CUDA kernels + the
extern "C" ABI in include/turboquant_c.h, + the C++ `turboquant::` API in
include/turboquant.h). `gemma4metal_b200.turboquant` is the Python mirror of
the reference's lib/turboquant.h over that ABI (ctypes; torch only for device
memory and streams).
"""
from .turboquant import load_library, version  # noqa: F401

__all__ = ["load_library", "version"]
