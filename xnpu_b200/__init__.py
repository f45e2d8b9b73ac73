"""xnpu_b200 -- B200-native (sm_100a) int4 ("w4" / Q4NX) weight path of xnpu.

The compute lives in libxq4.so (C ABI: include/xq4.h); this package is the
host-side mirror of the reference HAL's operator surface (see ``hal``) plus
seeded synthetic inputs (``synth``).
"""
from ._lib import Xq4Error, lib, LIB_PATH  # noqa: F401
from . import hal  # noqa: F401

__all__ = ["hal", "Xq4Error", "lib", "LIB_PATH"]
