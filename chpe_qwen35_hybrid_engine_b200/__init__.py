"""B200-native (sm_100a) quantized dequant-matmul path of the CHPE engine.

The compute lives in libchpe_b200.so (csrc/, C ABI in include/chpe_b200.h);
this package is the Python host mirror of the reference operator layer.
"""
from ._lib import ChpeError, load  # noqa: F401
from ._lib import (SCHEME_I8_GROUP_F16, SCHEME_I8_TENSOR, SCHEME_ROW_AFFINE_F32,  # noqa: F401
                   SCHEME_U_GROUP_F16_CONST_ZERO, SCHEME_U_GROUP_F16_ZERO, SCHEME_W2_CODEBOOK_GROUP_F16, X_BF16,
                   X_F16, X_F32, X_I8)
from .ops import Context, Tensor, kernel_launches  # noqa: F401

__all__ = ["Context", "Tensor", "ChpeError", "load"]
