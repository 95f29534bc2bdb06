"""novamlx_b200 — sm_100a implementation of NovaMLX's quantized decode/prefill hot path.

The compute lives in libnovamlx_cuda.so (C ABI: include/nmx.h); this package
holds its build script and a ctypes binding. Importing ``novamlx_b200.nmx``
loads the library and raises if it has not been built.
"""

__all__ = ["nmx"]
