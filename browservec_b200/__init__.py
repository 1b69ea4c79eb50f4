"""browservec_b200 -- B200-native (sm_100a) quantized flat-scan path of BrowserVec.

The CUDA library ``libbvcuda.so`` (C ABI in ``include/browservec.h``) holds the
kernels; this package is the Python host above it, mirroring the reference's
``VectorIndex`` seam (``AddonQuantIndex``) and the quantized branch of
``BrowserVec`` (``BrowserVec``).  There is no CPU fallback: importing the
index classes without the built library raises.
"""
from .index import AddonQuantIndex, BrowserVec, FlatHit, QueryResult  # noqa: F401
from .filter import compile_filter  # noqa: F401

__all__ = ["AddonQuantIndex", "BrowserVec", "FlatHit", "QueryResult", "compile_filter"]
