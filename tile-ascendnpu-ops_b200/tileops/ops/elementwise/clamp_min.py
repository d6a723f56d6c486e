"""ClampMinFwdOp -- lower-bound clamp, y = max(x, min), on the clamp kernel.

Same API as the reference op (ops/elementwise/clamp_min.py):
``ClampMinFwdOp(N_total, dtype, min=None, *, kernel_map=None)``; ``min`` is
required.  It reuses ``ClampScalarFwdKernel`` with ``max=None``.
"""

from __future__ import annotations

from typing import Dict, Optional

import torch

from tileops.kernels.elementwise.clamp_scalar import ClampScalarFwdKernel
from tileops.kernels.kernel_base import Kernel
from tileops.ops.elementwise._unary import UnaryFwdOp

__all__ = ["ClampMinFwdOp"]


class ClampMinFwdOp(UnaryFwdOp):
    """Element-wise ``clamp_min``; NaN propagates as in ``torch.clamp_min``.

    Args:
        N_total: Total number of elements (flattened input).
        dtype: float16, bfloat16 or float32.
        min: Lower bound (required).
        kernel_map: Optional kernel dispatch override.
    """

    _op_name = "clamp_min"
    kernel_cls = ClampScalarFwdKernel
    FLOPS_PER_ELEM = 1

    def __init__(
        self,
        N_total: int,
        dtype: torch.dtype,
        min: Optional[float] = None,
        *,
        kernel_map: Optional[Dict[str, Kernel]] = None,
    ):
        if min is None:
            raise ValueError("ClampMinFwdOp requires min")
        self.N_total = N_total
        self.dtype = dtype
        self.min = min
        self.max = None
        self.output_dtype = dtype
        self.dispatch_kernel(kernel_map)
        self.kernel = self.kernel_map[self._op_name](N_total, dtype, min, None)
