"""ClampScalarFwdOp -- scalar-bound clamp, y = clamp(x, min, max).

Same API as the reference op (ops/elementwise/clamp_scalar.py:30-111):
``ClampScalarFwdOp(N_total, dtype, min=None, max=None, *, kernel_map=None)``;
both bounds None raises ``ValueError("present(min) or present(max)")``.
"""

from __future__ import annotations

from typing import Dict, Optional

import torch

from tileops.kernels.elementwise.clamp_scalar import ClampScalarFwdKernel
from tileops.kernels.kernel_base import Kernel
from tileops.ops.elementwise._unary import UnaryFwdOp

__all__ = ["ClampScalarFwdOp"]


class ClampScalarFwdOp(UnaryFwdOp):
    """Element-wise clamp with scalar bounds; a ``None`` bound is not applied.

    Args:
        N_total: Total number of elements (flattened input).
        dtype: float16, bfloat16 or float32.
        min: Lower bound or None.
        max: Upper bound or None; at least one bound is given.
        kernel_map: Optional kernel dispatch override.
    """

    _op_name = "clamp_scalar"
    kernel_cls = ClampScalarFwdKernel
    # Manifest flops "1 * N": compare-and-select.
    FLOPS_PER_ELEM = 1

    def __init__(
        self,
        N_total: int,
        dtype: torch.dtype,
        min: Optional[float] = None,
        max: Optional[float] = None,
        *,
        kernel_map: Optional[Dict[str, Kernel]] = None,
    ):
        if min is None and max is None:
            raise ValueError("present(min) or present(max)")
        self.N_total = N_total
        self.dtype = dtype
        self.min = min
        self.max = max
        self.output_dtype = dtype
        self.dispatch_kernel(kernel_map)
        self.kernel = self.kernel_map[self._op_name](N_total, dtype, min, max)
