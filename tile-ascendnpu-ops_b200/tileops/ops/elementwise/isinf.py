"""IsinfFwdOp -- elementwise infinity predicate with a torch.bool output.

Same API as the reference op (ops/elementwise/isinf.py:36-115):
``IsinfFwdOp(N_total, dtype, *, kernel_map=None)`` over float16 / bfloat16 /
float32 inputs; other dtypes raise "does not support dtype".
"""

from __future__ import annotations

from typing import Dict, Optional

import torch

from tileops.kernels.elementwise.isinf import IsinfFwdKernel
from tileops.kernels.kernel_base import Kernel
from tileops.ops.elementwise._unary import UnaryFwdOp, reject_dtype

__all__ = ["IsinfFwdOp"]


class IsinfFwdOp(UnaryFwdOp):
    """Element-wise ``isinf(x)`` (bool output) on a flattened input.

    Args:
        N_total: Total number of elements (flattened input).
        dtype: Input dtype (float16, bfloat16 or float32).
        kernel_map: Optional kernel dispatch override.
    """

    _op_name = "isinf"
    kernel_cls = IsinfFwdKernel
    # Manifest flops "prod(S)": one predicate per element.
    FLOPS_PER_ELEM = 1
    _SUPPORTED_DTYPES = (torch.float16, torch.bfloat16, torch.float32)

    def __init__(
        self,
        N_total: int,
        dtype: torch.dtype,
        *,
        kernel_map: Optional[Dict[str, Kernel]] = None,
    ):
        reject_dtype("IsinfFwdOp", dtype, self._SUPPORTED_DTYPES)
        self.N_total = N_total
        self.dtype = dtype
        self.output_dtype = torch.bool
        self.dispatch_kernel(kernel_map)
        self.kernel = self.kernel_map[self._op_name](N_total, dtype)
