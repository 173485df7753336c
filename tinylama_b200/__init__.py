"""tinylama_b200 -- B200 (sm_100a) attention hot path for tinylama behind a C ABI.

The product is libtlattn.so (CUDA kernels + the C ABI in include/tl_attn.h).  This package
holds its build recipe (tinylama_b200.build), a ctypes binding (tinylama_b200._lib) and a
Python mirror of the reference's Nim procs (tinylama_b200.forward_attn) used by the tests
and the benchmark.  Importing the binding fails loudly when the library is not built.
"""
__all__ = ["forward_attn"]
