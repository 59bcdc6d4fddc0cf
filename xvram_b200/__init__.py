"""xvram_b200 -- B200-native out-of-core FP32 SGEMM behind xVRAM's C ABI.

The product is the native library ``xvram_b200/lib/libxvram_cuda_compat.so``
(C ABI: ``include/xvram_cuda_compat.h``, ``include/xvram_b200.h``).  This package
only binds it for Python callers, tests and the benchmark:

* ``xvram_b200.compat``  -- the cudaMalloc/cudaMemcpy/cublasSgemm-style table;
* ``xvram_b200.device``  -- the tile contraction on torch device tensors, the
  synthetic input generator, planner inspection and the FP32 peak probe.

Importing either submodule loads the library and raises ImportError when it has not
been built (``python -m xvram_b200.build``); there is no fallback implementation.
"""
from __future__ import annotations

__all__ = ["compat", "device"]
__version__ = "0.1.0"
