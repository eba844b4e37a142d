"""B200-native (sm_100a) forward of path-ordered geometric attention.

Drop-in for SiddhiMali/HolonomyAwareAttention's PathOrderedGeometricMHA
(core/attention.py, core/attention_fast_chunked.py): same constructor,
parameters and forward signature; the causal forward runs in hand-written
CUDA kernels behind the C ABI of libhoa.so (include/hoa.h).
"""
from .attention import PathOrderedGeometricMHA
from . import ops

__all__ = ["PathOrderedGeometricMHA", "ops"]
