"""Workloads of the norm family (reference workloads/norm.py:36-59)."""

import torch

from tileops.device import get_device_backend
from tileops.workloads.workload_base import WorkloadBase


class FusedAddLayerNormWorkload(WorkloadBase):
    """x / residual ``(m, n)`` and affine weight / bias ``(n,)``, all randn.

    ``affine_dtype`` (default: the input dtype, the reference contract) lets a
    benchmark draw float32 LayerNorm parameters.
    """

    def __init__(self, m: int, n: int, dtype: torch.dtype, eps: float = 1e-5,
                 affine_dtype: torch.dtype | None = None):
        self.m = m
        self.n = n
        self.dtype = dtype
        self.eps = eps
        self.affine_dtype = affine_dtype or dtype

    def gen_inputs(self) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
        device = get_device_backend().name
        x = torch.randn(self.m, self.n, dtype=self.dtype, device=device)
        residual = torch.randn(self.m, self.n, dtype=self.dtype, device=device)
        weight = torch.randn(self.n, dtype=self.affine_dtype, device=device)
        bias = torch.randn(self.n, dtype=self.affine_dtype, device=device)
        return x, residual, weight, bias
