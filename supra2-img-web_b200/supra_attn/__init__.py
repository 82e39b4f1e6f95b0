"""supra_attn — B200 (sm_100a) fused attention for Supra2-Img, behind the C ABI libsupra_attn.

The Python surface mirrors the reference's operator and runtime (app/gpu/ops.js:103-149,
app/gpu/device.js); see ops.py. Importing this package loads libsupra_attn.so and raises
ImportError if it has not been built; there is no fallback implementation.
"""

from ._lib import LIB_PATH, SupraAttnError, SupraAttnValueError, Desc, LinearDesc, SIGNATURES, lib
from .ops import (GPU, Tensor, attention, make_desc, linear, make_linear_desc, position_bias, relative_bucket,
                  default_scale)

__all__ = [
    "LIB_PATH",
    "SupraAttnError",
    "SupraAttnValueError",
    "Desc",
    "LinearDesc",
    "SIGNATURES",
    "lib",
    "GPU",
    "Tensor",
    "attention",
    "make_desc",
    "linear",
    "make_linear_desc",
    "position_bias",
    "relative_bucket",
    "default_scale",
]
