"""Workloads of the linear-attention family: Gated DeltaNet prefill, GLA decode.

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


class GLADecodeWorkload(WorkloadBase):
    """Single-token GLA decode workload (layout BHD), the reference's draws
    (examples/TileOPs/tileops/workloads/linear_attention.py:38-47): q, k, v
    ~ 0.5 N(0, 1), gk ~ -U(0, 1), state ~ N(0, 1), all in ``dtype``."""

    def __init__(self, B: int, H: int, DK: int, DV: int, dtype: torch.dtype,
                 scale: float = -1.0, device=None) -> None:
        self.B, self.H, self.DK, self.DV = B, H, DK, DV
        self.dtype = dtype
        self.scale = float(scale) if scale is not None and scale > 0 else DK ** -0.5
        self.device = device

    def gen_inputs(self):
        device = self.device or get_device_backend().name
        B, H, DK, DV, dt = self.B, self.H, self.DK, self.DV, self.dtype
        q = (torch.randn(B, H, DK, device=device, dtype=dt) * 0.5).contiguous()
        k = (torch.randn(B, H, DK, device=device, dtype=dt) * 0.5).contiguous()
        v = (torch.randn(B, H, DV, device=device, dtype=dt) * 0.5).contiguous()
        gk = (-torch.rand(B, H, DK, device=device, dtype=dt)).contiguous()
        state = torch.randn(B, H, DK, DV, device=device, dtype=dt).contiguous()
        return q, k, v, gk, state


def gla_decode_tolerance(dtype: torch.dtype) -> dict:
    """The reference's tolerance against the fp32 golden
    (examples/TileOPs/tileops/workloads/linear_attention.py:67-73)."""
    if dtype == torch.float16:
        return {"atol": 2e-3, "rtol": 2e-3}
    if dtype == torch.bfloat16:
        return {"atol": 2e-2, "rtol": 2e-2}
    return {"atol": 1e-4, "rtol": 1e-4}
