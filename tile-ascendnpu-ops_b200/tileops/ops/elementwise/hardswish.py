"""HardswishFwdOp -- elementwise HardSwish, y = x * clamp(x + 3, 0, 6) / 6.

Same API as the reference op (ops/elementwise/hardswish.py:27-107):
``HardswishFwdOp(N_total, dtype, inplace=False, *, kernel_map=None)``.
"""

from __future__ import annotations

from typing import Dict, Optional

import torch

from tileops.kernels.elementwise.hardswish import HardswishFwdKernel
from tileops.kernels.kernel_base import Kernel
from tileops.ops.elementwise._unary import UnaryFwdOp

__all__ = ["HardswishFwdOp"]


class HardswishFwdOp(UnaryFwdOp):
    """Element-wise HardSwish on a flattened input of ``N_total`` elements.

    Args:
        N_total: Total number of elements (flattened input).
        dtype: float16, bfloat16 or float32.
        inplace: When True, copy the result into ``input`` and return it.
        kernel_map: Optional kernel dispatch override.
    """

    _op_name = "hardswish"
    kernel_cls = HardswishFwdKernel
    # Manifest flops "4 * N": add, two-sided clamp, mul, div.
    FLOPS_PER_ELEM = 4

    def __init__(
        self,
        N_total: int,
        dtype: torch.dtype,
        inplace: bool = False,
        *,
        kernel_map: Optional[Dict[str, Kernel]] = None,
    ):
        self.N_total = N_total
        self.dtype = dtype
        self.inplace = inplace
        self.output_dtype = dtype
        self.dispatch_kernel(kernel_map)
        self.kernel = self.kernel_map[self._op_name](N_total, dtype)
