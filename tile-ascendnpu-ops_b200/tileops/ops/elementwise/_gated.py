"""Shared flow of the fused gated ops (GeluAndMul, GeluTanhAndMul).

Reference: ops/elementwise/gelu_and_mul.py:63-125 and
ops/elementwise/gelu_tanh_and_mul.py:43-126.  ``x`` has shape ``(M, 2N)``:
``gate = x[:, :N]``, ``value = x[:, N:]``; the output is ``(M, N)``.
Only float dtypes are admitted ("does not support dtype"); ``forward``
checks device, dtype ("x.dtype") and shape ("x.shape") before launching.
"""

from __future__ import annotations

from typing import Dict, Optional

import torch

from tileops.device import get_device_backend
from tileops.kernels.kernel_base import Kernel
from tileops.ops.elementwise._unary import reject_dtype
from tileops.ops.op_base import Op


class GatedFwdOp(Op):
    _op_name: str = ""
    kernel_cls: type = None
    FLOPS_PER_OUTPUT: int = 1
    _SUPPORTED_DTYPES = (torch.float16, torch.bfloat16, torch.float32)

    def __init__(
        self,
        M: int,
        N: int,
        dtype: torch.dtype,
        *,
        kernel_map: Optional[Dict[str, Kernel]] = None,
    ):
        reject_dtype(type(self).__name__, dtype, self._SUPPORTED_DTYPES)
        self.M = int(M)
        self.N = int(N)
        self.dtype = dtype
        self.output_dtype = dtype
        self.x_shape = (self.M, 2 * self.N)
        self.out_shape = (self.M, self.N)
        self.N_total = self.M * self.N
        self.dispatch_kernel(kernel_map)
        self.kernel = self.kernel_map[self._op_name](self.M, self.N, dtype)

    @property
    def default_kernel_map(self) -> Dict[str, Kernel]:
        return {self._op_name: self.kernel_cls}

    def _validate_input(self, x: torch.Tensor) -> None:
        backend = get_device_backend()
        if not backend.is_device_tensor(x):
            raise ValueError(f"x must be a {backend.name} tensor, got device {x.device}")
        if x.dtype != self.dtype:
            raise ValueError(f"Expected x.dtype {self.dtype}, got {x.dtype}")
        if tuple(x.shape) != self.x_shape:
            raise ValueError(f"Expected x.shape {self.x_shape}, got {tuple(x.shape)}")

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x = x.contiguous()
        self._validate_input(x)
        return self.kernel(x)

    def eval_roofline(self) -> tuple[int, int]:
        """``(FLOPS_PER_OUTPUT * M * N, 3 * M * N * elem_bytes)``."""
        return self.FLOPS_PER_OUTPUT * self.N_total, 3 * self.N_total * self.dtype.itemsize
