"""GLADecodeOp (single-token gated linear attention decode).

Same class as the reference (examples/TileOPs/tileops/ops/linear_attention/
gla_decode.py:24-77): layout BHD, one recurrent step per call,

    state_new[dk, dv] = exp(gk[dk]) * state[dk, dv] + k[dk] * v[dv]
    o[dv]             = scale * sum_dk q[dk] * state_new[dk, dv]

``scale`` is fixed at construction (non-positive means ``DK ** -0.5``); the
state is returned functionally as ``new_state``.  Unlike the reference, the
input shapes and dtypes are checked before the launch (the native kernel
trusts its sizes).
"""

from typing import Dict, Optional

import torch

from tileops.device import get_device_backend
from tileops.kernels.kernel_base import Kernel
from tileops.kernels.linear_attention.gla_decode import GLADecodeKernel
from tileops.ops.op_base import Op

__all__ = ["GLADecodeOp"]


class GLADecodeOp(Op):
    """Single-step (decode) gated linear attention, layout BHD.

    Args:
        B, H, DK, DV: batch / heads / key-dim / value-dim.
        scale: readout scale; non-positive means ``DK ** -0.5``.
        dtype: float16 / bfloat16 / float32.
        k_tile: optional DK sub-tile override (kept as a config entry).
        kernel_map: optional override for kernel dispatch.
    """

    def __init__(self, B: int, H: int, DK: int, DV: int, scale: float = -1.0,
                 dtype: torch.dtype = torch.bfloat16, k_tile: Optional[int] = None,
                 kernel_map: Optional[Dict[str, Kernel]] = None) -> None:
        self.B = B
        self.H = H
        self.DK = DK
        self.DV = DV
        self.scale = scale
        self.dtype = dtype
        self.dispatch_kernel(kernel_map)
        self.kernel: Kernel = self.kernel_map["gla_decode"](B, H, DK, DV, dtype, scale, k_tile)

    @property
    def default_kernel_map(self) -> Dict[str, Kernel]:
        return {"gla_decode": GLADecodeKernel}

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, gk: torch.Tensor,
                state: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """Run one decode step; returns ``(o, new_state)``."""
        backend = get_device_backend()
        B, H, DK, DV = self.B, self.H, self.DK, self.DV
        for name, t, shape in (("q", q, (B, H, DK)), ("k", k, (B, H, DK)), ("v", v, (B, H, DV)),
                               ("gk", gk, (B, H, DK)), ("state", state, (B, H, DK, DV))):
            if not backend.is_device_tensor(t):
                raise ValueError(f"{name} must be a {backend.name} tensor, got device {t.device}")
            if tuple(t.shape) != shape:
                raise ValueError(f"Expected {name}.shape {shape}, got {tuple(t.shape)}")
            if t.dtype != self.dtype:
                raise ValueError(f"Expected {name}.dtype {self.dtype}, got {t.dtype}")
        return self.kernel(q, k, v, gk, state)

    def eval_roofline(self) -> tuple[int, int]:
        """Return ``(flops, bytes)`` for ``B*H*(5*DK*DV + DK + DV)`` FLOPs."""
        elem_bytes = self.dtype.itemsize
        flops = self.B * self.H * (5 * self.DK * self.DV + self.DK + self.DV)
        nbytes = self.B * self.H * (3 * self.DK + 2 * self.DV + 2 * self.DK * self.DV)
        return int(flops), int(nbytes * elem_bytes)
