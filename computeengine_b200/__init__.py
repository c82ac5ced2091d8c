"""B200-native Conv2D forward backend for ComputeEngine (fp32 and int8).

Native code lives in libie_cuda_conv.so (hand-written sm_100a kernels behind
the C ABI in include/ie_cuda_conv.h); this package binds it (``_lib``) and
mirrors the reference engine's operator interface (``ops``).
"""
import torch  # noqa: F401  (loads the CUDA runtime before the native library)

__all__ = ["ops", "quant", "resnet"]
