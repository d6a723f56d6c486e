"""Workloads of the linear-attention family: Gated DeltaNet prefill.

Inputs in BTHD layout with the distributions of the benchmark configuration:
q, k ~ N(0, 1) L2-normalised per head (in fp32, then cast), v ~ N(0, 1),
g = logsigmoid(N(0, 1)) / 16 (per-token log decay), beta = sigmoid(N(0, 1)).
"""

import torch
import torch.nn.functional as F

from tileops.device import get_device_backend
from tileops.workloads.workload_base import WorkloadBase


class GdnPrefillWorkload(WorkloadBase):
    def __init__(self, batch: int, seq_len: int, heads: int, dim_k: int, dim_v: int,
                 dtype: torch.dtype = torch.bfloat16, device=None):
        self.batch, self.seq_len, self.heads = batch, seq_len, heads
        self.dim_k, self.dim_v, self.dtype = dim_k, dim_v, dtype
        self.device = device

    def gen_inputs(self):
        device = self.device or get_device_backend().name
        B, T, H = self.batch, self.seq_len, self.heads
        q = F.normalize(torch.randn(B, T, H, self.dim_k, device=device), dim=-1).to(self.dtype)
        k = F.normalize(torch.randn(B, T, H, self.dim_k, device=device), dim=-1).to(self.dtype)
        v = torch.randn(B, T, H, self.dim_v, device=device).to(self.dtype)
        g = F.logsigmoid(torch.randn(B, T, H, device=device)) / 16
        beta = torch.sigmoid(torch.randn(B, T, H, device=device))
        return q, k, v, g, beta
