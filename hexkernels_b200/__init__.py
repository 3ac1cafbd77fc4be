"""hexkernels_b200: B200-native (sm_100a) implementation of the hexkernels
corpus's DL-operator hot path.

The product is the C ABI in include/hexcuda.h (libhexcuda.so, built in-tree)
and the candidate_kernel shims in shims/ that let the corpus's own harness.c
files link unchanged.  This Python package is host plumbing over that ABI:
``ops`` (NumPy in/out through the host-pointer entries) and ``device`` (device
pointers, e.g. torch tensors, through the asynchronous launchers).
"""
from ._lib import HexcudaError, LIB_PATH, load  # noqa: F401

__all__ = ["HexcudaError", "LIB_PATH", "load"]
