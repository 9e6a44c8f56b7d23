"""aljabr_b200 -- B200 (sm_100a) provider for Aljabr's quantized decode path.

The compute lives in libaljabr_blackwell.so (hand-written CUDA kernels behind
the C-ABI in include/aljabr_blackwell.h).  This package holds its ctypes
binding (`native`), host-side mirrors of the reference's dispatch seam and
provider SPI (`bridge`, `provider`), and the build step (`build`).
"""
from . import native  # noqa: F401

__all__ = ["native"]
