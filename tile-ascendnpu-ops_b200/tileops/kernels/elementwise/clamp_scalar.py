"""ClampScalarFwdKernel: y = clamp(x, min, max) with scalar bounds.

Replaces kernels/elementwise/clamp_scalar/clamp_scalar.py:82 (TileLang
clamp_scalar_fwd_kernel) with tileops_clamp_scalar_fwd.  The comparison runs
in fp32 with the bounds rounded to fp32; NaN propagates as in torch.clamp.
"""

from typing import Optional

import torch

from tileops.kernels.elementwise._unary import FLOAT_DTYPES, UnaryNativeKernel
from tileops.kernels.kernel_base import check_dtype

__all__ = ["ClampScalarFwdKernel"]


class ClampScalarFwdKernel(UnaryNativeKernel):
    """Scalar-bound clamp; a ``None`` bound is not applied.

    Args:
        N_total: Total number of elements (flattened input).
        dtype: float16, bfloat16 or float32.
        min_val: Lower bound or None.
        max_val: Upper bound or None (at least one bound is required).
        config: Optional config dict (no tunables).
    """

    SUPPORTED_DTYPES = FLOAT_DTYPES
    entry_point = "tileops_clamp_scalar_fwd"

    def __init__(
        self,
        N_total: int,
        dtype: torch.dtype,
        min_val: Optional[float] = None,
        max_val: Optional[float] = None,
        config: Optional[dict] = None,
    ):
        if min_val is None and max_val is None:
            raise ValueError("ClampScalarFwdKernel requires present(min) or present(max)")
        check_dtype(self, dtype, self.SUPPORTED_DTYPES)
        self.min_val = min_val
        self.max_val = max_val
        super().__init__(N_total, dtype, config)

    def _scalar_args(self) -> tuple:
        return (
            int(self.min_val is not None),
            float(self.min_val if self.min_val is not None else 0.0),
            int(self.max_val is not None),
            float(self.max_val if self.max_val is not None else 0.0),
        )
