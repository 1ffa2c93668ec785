"""ternative_b200 -- B200-native (sm_100a) quantized-weight hot path for ternative.

The product is libtvb200.so (C ABI in include/tvb200.h, CUDA in csrc/).  This
package is its Python host side: a ctypes binding, a mirror of the reference's
CUDABackend class, and the model-level driver used by the tests and bench.
"""
from ._lib import (TVB_F16, TVB_F32, TVB_I8_ROW, TVB_I8_TENSOR, MergeDesc, TvbError, load)
from .backend import Config, CUDABackend, DeviceWeight

__all__ = ["TVB_F16", "TVB_F32", "TVB_I8_ROW", "TVB_I8_TENSOR", "MergeDesc", "TvbError", "load",
           "Config", "CUDABackend", "DeviceWeight"]
