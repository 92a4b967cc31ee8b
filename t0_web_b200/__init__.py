"""B200-native (sm_100a) engine for t0-web's quantized t0-alpha forecast path.

The product is libt0b.so (CUDA kernels + C ABI, include/t0b.h); this package
is its Python host mirror of the reference `t0_fast` API.
"""
from . import gguf, synthetic, t0_fast  # noqa: F401
from ._lib import LIB_PATH, T0bError  # noqa: F401
