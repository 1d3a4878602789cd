"""alpaka3_b200: B200-native (sm_100a) implementation of alpaka3's data-parallel primitive path.

The product is the CUDA library ``lib/libalpaka3_b200.so`` behind the C ABI in ``include/alpaka3_b200.h`` and the
C++20 alpaka-shaped front end in ``include/alpaka3_b200/``. This Python package is the binding used by the tests, the
benchmark and the multi-GPU driver: :mod:`.capi` (ctypes declarations), :mod:`.algo` (onHost-style calls on torch
device tensors) and :mod:`.dist` (sharding over one process per GPU).
"""
__version__ = "0.1.0"
