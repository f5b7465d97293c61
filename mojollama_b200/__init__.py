"""mojollama_b200 -- B200-native (sm_100a) drop-in for MojoLlama's C-engine hot path.

The product is the native library ``lib/libmojollama_b200.so`` and its
reference-named alias libraries (``combined_engine.so``, ``simd_ops.so``,
``gqa_attention.so``, ...), which the reference's Python engines load through
ctypes unchanged.  This Python package is the thin host side:

  _lib       ctypes loader (fails loudly when the libraries are missing)
  kernels    the reference's ctypes bindings, restated against the alias libraries
  ops        torch-friendly wrappers over the mlq_* C-ABI (device tensors)
  build      in-tree build of the native libraries
"""
from ._lib import LIB_DIR, NativeLibraryMissing, check, core, load_alias  # noqa: F401

__all__ = ["LIB_DIR", "NativeLibraryMissing", "check", "core", "load_alias"]
