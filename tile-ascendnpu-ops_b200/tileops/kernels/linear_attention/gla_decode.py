"""GLADecodeKernel: gated linear attention, one decode step (layout BHD).

Native entry point ``tileops_gla_decode_fwd``: one CTA per (batch, head) and
slice of the value columns, the state read and written once in 16-byte
packets with fp32 math.  Replaces the reference factory
kernels/linear_attention/gla_decode/gla_decode_kernel/_gla_decode_kernel.py:57
behind the same class (kernels/linear_attention/gla_decode/gla_decode.py:23-68):
same constructor, ``scale`` resolution (non-positive -> ``DK ** -0.5``),
``k_tile`` config entry and outputs ``(o, new_state)`` in the input dtype.
"""

from __future__ import annotations

from typing import Optional

import torch

from tileops import _native
from tileops.kernels.kernel_base import Kernel, check_dtype

__all__ = ["GLADecodeKernel"]


def _ceil_ktile_fit(dk: int, dv: int) -> int:
    """The reference's default DK sub-tile (its on-chip buffer fit rule,
    _gla_decode_kernel.py:44-54); kept as the ``k_tile`` config value.  The
    CUDA kernel streams rows and has no such tile."""
    for kt in (32, 16, 8, 4, 2, 1):
        if dk % kt:
            continue
        if 9 * kt * dv * 4 + 2 * kt * dv * 2 <= 150 * 1024:
            return kt
    return 1


class GLADecodeKernel(Kernel):
    """Single-step (decode) gated linear attention, layout BHD."""

    supported_archs: Optional[list] = [100]
    SUPPORTED_DTYPES = (torch.float16, torch.bfloat16, torch.float32)

    def __init__(self, B: int, H: int, DK: int, DV: int, dtype: torch.dtype = torch.bfloat16,
                 scale: float = -1.0, k_tile: Optional[int] = None,
                 config: Optional[dict] = None) -> None:
        super().__init__()
        check_dtype(self, dtype, self.SUPPORTED_DTYPES)
        self.B, self.H, self.DK, self.DV = B, H, DK, DV
        self.dtype = dtype
        self.scale = float(scale) if scale is not None and scale > 0 else DK ** -0.5
        if k_tile is None:
            k_tile = _ceil_ktile_fit(DK, DV)
        if DK % k_tile:
            raise ValueError(f"DK ({DK}) must be divisible by k_tile ({k_tile})")
        self.k_tile = k_tile
        self.init_config(config)

    @property
    def default_config(self) -> dict:
        return {"k_tile": self.k_tile}

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, gk: torch.Tensor,
                state: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        q, k, v, gk, state = (t.contiguous() for t in (q, k, v, gk, state))
        o = torch.empty((self.B, self.H, self.DV), dtype=self.dtype, device=q.device)
        new_state = torch.empty((self.B, self.H, self.DK, self.DV), dtype=self.dtype,
                                device=q.device)
        _native.launch(
            "tileops_gla_decode_fwd", q.device,
            _native.ptr(q), _native.ptr(k), _native.ptr(v), _native.ptr(gk), _native.ptr(state),
            _native.ptr(o), _native.ptr(new_state),
            self.B, self.H, self.DK, self.DV, float(self.scale), _native.dtype_code(self.dtype),
        )
        return o, new_state
