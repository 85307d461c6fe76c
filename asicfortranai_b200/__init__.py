"""asicfortranai_b200 -- B200 (sm_100a) implementation of asicForTranAI's quantized
matmul hot path (3.5-bit / INT4 weights, int8 activations, exact int32 accumulation)
and the LLaMA decode loop on top of it.

The compute lives in libq35.so (CUDA for sm_100a, C ABI in include/q35.h); this package
is the Python mirror of the reference's Fortran module interfaces over that library.
"""
from . import _lib  # noqa: F401
from ._lib import Q35Error, Q35_FMT_3P5BIT, Q35_FMT_INT4  # noqa: F401

__all__ = ["Q35Error", "Q35_FMT_3P5BIT", "Q35_FMT_INT4"]
