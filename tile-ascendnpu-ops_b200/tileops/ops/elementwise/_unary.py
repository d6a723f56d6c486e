"""Shared flow of the flat elementwise ops.

Every reference unary op (e.g. ops/elementwise/hardswish.py:27-107,
ops/elementwise/isnan.py:36-115) validates the input (device, dtype, element
count), flattens ``input.contiguous().reshape(-1)``, runs the kernel and
reshapes back; ``eval_roofline`` is ``(FLOPS_PER_ELEM * N, N * (in + out
elem bytes))``.  Subclasses define the constructor (its parameter names are
the reconstruction contract of ``_extract_op_init_args``), ``_op_name``,
``kernel_cls`` and ``FLOPS_PER_ELEM``.
"""

from __future__ import annotations

from typing import Dict

import torch

from tileops.device import get_device_backend
from tileops.kernels.kernel_base import Kernel
from tileops.ops.op_base import Op


class UnaryFwdOp(Op):
    _op_name: str = ""
    kernel_cls: type = None
    FLOPS_PER_ELEM: int = 1
    inplace: bool = False

    @property
    def default_kernel_map(self) -> Dict[str, Kernel]:
        return {self._op_name: self.kernel_cls}

    def _validate_input(self, input: torch.Tensor) -> None:
        backend = get_device_backend()
        if not backend.is_device_tensor(input):
            raise ValueError(f"input must be a {backend.name} tensor, got device {input.device}")
        if input.dtype != self.dtype:
            raise ValueError(f"Expected input.dtype {self.dtype}, got {input.dtype}")
        if input.numel() != self.N_total:
            raise ValueError(f"Expected {self.N_total} elements, got {input.numel()}")

    def _eager_forward(self, input: torch.Tensor) -> torch.Tensor:
        """Flatten -> kernel -> reshape."""
        orig_shape = input.shape
        flat = input.contiguous().reshape(-1)
        return self.kernel(flat).reshape(orig_shape)

    def forward(self, input: torch.Tensor) -> torch.Tensor:
        self._validate_input(input)
        if self.inplace:
            result = self._eager_forward(input)
            input.copy_(result.reshape(input.shape))
            return input
        return self._eager_forward(input)

    @property
    def total_memory(self) -> float:
        """Read x + write y."""
        return self.N_total * (self.dtype.itemsize + self.output_dtype.itemsize)

    def eval_roofline(self) -> tuple[int, int]:
        """``(FLOPS_PER_ELEM * N, N * (input elem bytes + output elem bytes))``."""
        return self.FLOPS_PER_ELEM * self.N_total, int(self.total_memory)


def reject_dtype(op_name: str, dtype: torch.dtype, supported: tuple) -> None:
    """The reference's op-level dtype error."""
    if dtype not in supported:
        names = ", ".join(str(dt) for dt in supported)
        raise ValueError(f"{op_name} does not support dtype {dtype}. Supported: [{names}]")
