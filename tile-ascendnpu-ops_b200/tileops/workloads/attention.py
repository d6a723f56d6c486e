"""Workloads of the attention family (reference workloads/attention.py:22-51)."""

import torch

from tileops.device import get_device_backend
from tileops.workloads.workload_base import WorkloadBase

__all__ = ["MhaFwdWorkload"]


class MhaFwdWorkload(WorkloadBase):
    """q / k / v in BSHD layout, each ``(batch, seq_len, heads, dim)`` randn."""

    def __init__(self, batch: int, heads: int, seq_len: int, dim: int, is_causal: bool,
                 dtype: torch.dtype):
        self.batch = batch
        self.heads = heads
        self.seq_len = seq_len
        self.dim = dim
        self.is_causal = is_causal
        self.dtype = dtype

    def gen_inputs(self) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        device = get_device_backend().name
        shape = (self.batch, self.seq_len, self.heads, self.dim)
        q = torch.randn(*shape, device=device, dtype=self.dtype)
        k = torch.randn(*shape, device=device, dtype=self.dtype)
        v = torch.randn(*shape, device=device, dtype=self.dtype)
        return q, k, v
