"""Mamba-2 State-Space Dual (SSD) fused chunk output operator.

Same class as the reference (examples/TileOPs/tileops/ops/mamba/ssd_chunk_scan.py:29-213):
constructed with only a ``kernel_map``; the shapes are bound by ``forward``
(kernels cached per shape and device), computing

  out[l, p] = exp(dA_cumsum[l]) * (C[l] @ prev_states)
            + sum_{s <= l} cb[l, s] * exp(dA_cumsum[l] - dA_cumsum[s]) * dt[s] * x[s, p]

``eval_roofline`` raises before the first ``forward``, as there.  Besides the
reference's shape checks, dtypes are checked before the launch (the native
kernel trusts its sizes).
"""

from __future__ import annotations

from typing import Dict, Optional

import torch

from tileops.device import get_device_backend
from tileops.kernels.kernel_base import Kernel
from tileops.kernels.mamba import SSDChunkScanFwdKernel
from tileops.ops.op_base import Op

__all__ = ["SSDChunkScanFwdOp"]


class SSDChunkScanFwdOp(Op):
    """Mamba-2 State-Space Dual (SSD) fused chunk output operator.

    Args:
        kernel_map: Optional override for kernel dispatch.
    """

    def __init__(self, kernel_map: Optional[Dict[str, Kernel]] = None):
        self.batch = None
        self.num_chunks = None
        self.chunk_len = None
        self.n_heads = None
        self.d_head = None
        self.d_state = None
        self.n_groups = None
        self.dtype = None
        self.dispatch_kernel(kernel_map)
        self._kernel_cache: Dict[tuple, Kernel] = {}
        self.kernel = None

    @property
    def default_kernel_map(self) -> Dict[str, Kernel]:
        return {"ssd_chunk_scan_fwd": SSDChunkScanFwdKernel}

    def _get_kernel(self, batch, num_chunks, chunk_len, n_heads, d_head, d_state, n_groups,
                    dtype, device_index) -> Kernel:
        key = (batch, num_chunks, chunk_len, n_heads, d_head, d_state, n_groups, dtype,
               device_index)
        if key not in self._kernel_cache:
            self._kernel_cache[key] = self.kernel_map["ssd_chunk_scan_fwd"](
                batch, num_chunks, chunk_len, n_heads, d_head, d_state, n_groups, dtype)
        return self._kernel_cache[key]

    def forward(self, x: torch.Tensor, cb: torch.Tensor, dA_cumsum: torch.Tensor,
                C: torch.Tensor, prev_states: torch.Tensor, dt: torch.Tensor) -> torch.Tensor:
        """x (B, S, H, P), cb (B, NC, G, Q, Q), dA_cumsum (B, H, NC, Q) fp32,
        C (B, S, G, N), prev_states (B, NC, H, P, N) fp32, dt (B, H, NC, Q);
        returns out (B, S, H, P) fp32."""
        backend = get_device_backend()
        if not backend.is_device_tensor(x):
            raise ValueError(f"x must be a {backend.name} tensor, got device {x.device}")
        if x.ndim != 4:
            raise ValueError("x must have shape [batch, seq_len, n_heads, d_head]")
        batch, seq_len, n_heads, d_head = x.shape
        if dA_cumsum.ndim != 4:
            raise ValueError("dA_cumsum must have shape [batch, n_heads, num_chunks, chunk_len]")
        if dA_cumsum.shape[0] != batch or dA_cumsum.shape[1] != n_heads:
            raise ValueError("dA_cumsum must match x batch and n_heads")
        num_chunks, chunk_len = dA_cumsum.shape[2], dA_cumsum.shape[3]
        if seq_len != num_chunks * chunk_len:
            raise ValueError("x seq_len must equal num_chunks * chunk_len")
        if C.ndim != 4 or C.shape[0] != batch or C.shape[1] != seq_len:
            raise ValueError("C must have shape [batch, seq_len, n_groups, d_state]")
        n_groups, d_state = C.shape[2], C.shape[3]
        if n_heads % n_groups != 0:
            raise ValueError("n_heads must be divisible by n_groups")
        if cb.shape != (batch, num_chunks, n_groups, chunk_len, chunk_len):
            raise ValueError(
                "cb must have shape [batch, num_chunks, n_groups, chunk_len, chunk_len]")
        if prev_states.shape != (batch, num_chunks, n_heads, d_head, d_state):
            raise ValueError(
                "prev_states must have shape [batch, num_chunks, n_heads, d_head, d_state]")
        if dt.shape != (batch, n_heads, num_chunks, chunk_len):
            raise ValueError("dt must have shape [batch, n_heads, num_chunks, chunk_len]")
        for name, t in (("cb", cb), ("dA_cumsum", dA_cumsum), ("C", C),
                        ("prev_states", prev_states), ("dt", dt)):
            if not backend.is_device_tensor(t) or t.device != x.device:
                raise ValueError(f"{name} must be a {backend.name} tensor on {x.device}")
        for name, t in (("cb", cb), ("C", C), ("dt", dt)):
            if t.dtype != x.dtype:
                raise ValueError(f"Expected {name}.dtype {x.dtype}, got {t.dtype}")

        self.batch = batch
        self.num_chunks = num_chunks
        self.chunk_len = chunk_len
        self.n_heads = n_heads
        self.d_head = d_head
        self.d_state = d_state
        self.n_groups = n_groups
        self.dtype = x.dtype
        self.kernel = self._get_kernel(batch, num_chunks, chunk_len, n_heads, d_head, d_state,
                                       n_groups, x.dtype, x.device.index)
        return self.kernel(x, cb, dA_cumsum, C, prev_states, dt)

    def eval_roofline(self) -> tuple[int, int]:
        """``(flops, bytes)``: history path ``2 * tokens * d_state * d_head``
        plus the intra-chunk path ``batch * num_chunks * n_heads * chunk_len**2 *
        d_head`` (the reference's formula, ssd_chunk_scan.py:180-213)."""
        if self.batch is None or self.dtype is None:
            raise RuntimeError(
                f"{type(self).__name__}.eval_roofline() requires a prior forward() "
                "call to bind dynamic input shape")
        batch, num_chunks, chunk_len = int(self.batch), int(self.num_chunks), int(self.chunk_len)
        n_heads, d_head, d_state = int(self.n_heads), int(self.d_head), int(self.d_state)
        n_groups = int(self.n_groups)
        elem_bytes = self.dtype.itemsize
        seq_len = num_chunks * chunk_len
        tokens = batch * seq_len * n_heads
        flops = (2 * tokens * d_state * d_head
                 + batch * num_chunks * n_heads * chunk_len**2 * d_head)
        nbytes = (tokens * d_head * elem_bytes
                  + batch * num_chunks * n_groups * chunk_len**2 * elem_bytes
                  + tokens * 4
                  + batch * seq_len * n_groups * d_state * elem_bytes
                  + batch * num_chunks * n_heads * d_head * d_state * 4
                  + tokens * elem_bytes
                  + tokens * d_head * 4)
        return int(flops), int(nbytes)
