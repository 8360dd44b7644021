"""fufft_b200: fused FFT convolution for NVIDIA B200 (sm_100a).

The product is the shared library libfufft_b200.so (C ABI in
include/fufft_b200.h, CUDA kernels in csrc/).  This package is its Python
front end: ``fufft_b200.ops`` mirrors the reference's entry points over CUDA
tensors; ``fufft_b200.build`` is the build recipe.
"""
from . import ops  # noqa: F401
from ._lib import FufftError, lib  # noqa: F401

__all__ = ["ops", "lib", "FufftError"]
