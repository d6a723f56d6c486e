"""BitwiseNotFwdOp -- elementwise bitwise NOT (~x; logical not for bool).

Same API as the reference op (ops/elementwise/bitwise_not.py:33-119):
``BitwiseNotFwdOp(N_total, dtype, *, kernel_map=None)`` over bool / uint8 /
int8 / int16 / int32 / int64.
"""

from __future__ import annotations

from typing import Dict, Optional

import torch

from tileops.kernels.elementwise.bitwise_not import BitwiseNotFwdKernel
from tileops.kernels.kernel_base import Kernel
from tileops.ops.elementwise._unary import UnaryFwdOp, reject_dtype

__all__ = ["BitwiseNotFwdOp"]


class BitwiseNotFwdOp(UnaryFwdOp):
    """Element-wise ``~x`` on a flattened input of ``N_total`` elements.

    Args:
        N_total: Total number of elements (flattened input).
        dtype: bool, uint8, int8, int16, int32 or int64.
        kernel_map: Optional kernel dispatch override.
    """

    _op_name = "bitwise_not"
    kernel_cls = BitwiseNotFwdKernel
    FLOPS_PER_ELEM = 1
    _SUPPORTED_DTYPES = (
        torch.bool,
        torch.uint8,
        torch.int8,
        torch.int16,
        torch.int32,
        torch.int64,
    )

    def __init__(
        self,
        N_total: int,
        dtype: torch.dtype,
        *,
        kernel_map: Optional[Dict[str, Kernel]] = None,
    ):
        reject_dtype("BitwiseNotFwdOp", dtype, self._SUPPORTED_DTYPES)
        self.N_total = N_total
        self.dtype = dtype
        self.output_dtype = dtype
        self.dispatch_kernel(kernel_map)
        self.kernel = self.kernel_map[self._op_name](N_total, dtype)
