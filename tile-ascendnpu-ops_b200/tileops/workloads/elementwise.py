"""Workloads of the elementwise family (reference workloads/elementwise.py).

Special-value draws follow the reference: the float predicates get a quarter
each of NaN, +Inf, -Inf and finite values (elementwise.py:85-173); bitwise
NOT draws bool ``rand > 0.5``, full-range uint8, or a small symmetric range
for the signed types (elementwise.py:51-82).
"""

from math import prod

import torch

from tileops.device import get_device_backend
from tileops.workloads.workload_base import RandnWorkload, WorkloadBase


class ShapedRandnWorkload(RandnWorkload):
    """One ``randn`` tensor of arbitrary rank, with its element count."""

    def __init__(self, shape: tuple, dtype):
        super().__init__(tuple(shape), dtype)
        self.n_total = prod(self.shape)


class HardsigmoidWorkload(ShapedRandnWorkload):
    """HardsigmoidFwdOp input."""


class HardswishWorkload(ShapedRandnWorkload):
    """HardswishFwdOp input."""


class ClampScalarWorkload(ShapedRandnWorkload):
    """ClampScalarFwdOp input (the bounds are op parameters)."""


class ClampMinWorkload(ShapedRandnWorkload):
    """ClampMinFwdOp input (the bound is an op parameter)."""


class BitwiseNotWorkload(WorkloadBase):
    """Bool / integer input for BitwiseNotFwdOp."""

    def __init__(self, shape: tuple[int, ...], dtype: torch.dtype):
        self.shape = tuple(shape)
        self.input_shape = self.shape
        self.n_total = prod(self.shape)
        self.dtype = dtype

    def gen_inputs(self) -> tuple[torch.Tensor]:
        device = get_device_backend().name
        if self.dtype == torch.bool:
            x = torch.rand(self.shape, device=device) > 0.5
        elif self.dtype == torch.uint8:
            x = torch.randint(0, 256, self.shape, device=device, dtype=self.dtype)
        else:
            lo = max(torch.iinfo(self.dtype).min, -128)
            hi = min(torch.iinfo(self.dtype).max, 128)
            x = torch.randint(lo, hi, self.shape, device=device, dtype=self.dtype)
        return (x,)


class _SpecialValueWorkload(WorkloadBase):
    """randn with the first three quarters set to NaN, +Inf and -Inf."""

    def __init__(self, shape: tuple[int, ...], dtype: torch.dtype):
        self.shape = tuple(shape)
        self.input_shape = self.shape
        self.n_total = prod(self.shape)
        self.dtype = dtype

    def gen_inputs(self) -> tuple[torch.Tensor]:
        device = get_device_backend().name
        x = torch.randn(self.shape, device=device, dtype=self.dtype)
        flat = x.view(-1)
        quarter = flat.numel() // 4
        flat[:quarter] = float("nan")
        flat[quarter : 2 * quarter] = float("inf")
        flat[2 * quarter : 3 * quarter] = float("-inf")
        return (x,)


class IsnanWorkload(_SpecialValueWorkload):
    """IsnanFwdOp input."""


class IsinfWorkload(_SpecialValueWorkload):
    """IsinfFwdOp input (the NaN quarter must read False)."""


class IsfiniteWorkload(_SpecialValueWorkload):
    """IsfiniteFwdOp input."""


class GatedWorkload(WorkloadBase):
    """One ``(M, 2N)`` randn tensor for the fused gated ops."""

    def __init__(self, M: int, N: int, dtype: torch.dtype):
        self.M = int(M)
        self.N = int(N)
        self.dtype = dtype
        self.x_shape = (self.M, 2 * self.N)

    def gen_inputs(self) -> tuple[torch.Tensor]:
        device = get_device_backend().name
        return (torch.randn(self.M, 2 * self.N, device=device, dtype=self.dtype),)
