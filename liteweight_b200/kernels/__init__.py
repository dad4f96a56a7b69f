"""Drop-in replacements of liteweight's ``kernels`` package (kernels/__init__.py:1-5).

Same names, signatures, dtype/shape assertions and output allocation as the
Triton originals; the work runs in the sm_100a CUDA library through its C ABI.
"""

from liteweight_b200.kernels.matmul_fp16 import matmul_fp16
from liteweight_b200.kernels.matmul_int4 import matmul_int4
from liteweight_b200.kernels.matmul_int8 import matmul_int8

__all__ = ["matmul_fp16", "matmul_int8", "matmul_int4"]
