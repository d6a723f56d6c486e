"""FusedAddLayerNormKernel: residual add + LayerNorm, two outputs.

Replaces kernels/norm/fused_add_layer_norm/fused_add_layer_norm.py:61-156
(TileLang _fused_add_layer_norm_kernel) with the native entry point
tileops_fused_add_layer_norm_fwd.  Per row of N::

    s = round_dtype(x + residual)                  # residual_out
    y = round_dtype((s - mean(s)) * rstd * weight + bias)

Statistics are fp32 (biased variance).  ``weight`` / ``bias`` may be the
input dtype (the reference contract) or float32.
"""

from typing import Optional

import torch

from tileops import _native
from tileops.kernels.kernel_base import Kernel, check_dtype

__all__ = ["FusedAddLayerNormKernel"]


class FusedAddLayerNormKernel(Kernel):
    """Fused Add + LayerNorm forward kernel.

    Args:
        M: Number of rows (product of all leading dims of ``x``).
        N: Hidden dimension (last dim of ``x``).
        eps: Epsilon for numerical stability.
        dtype: float32, float16 or bfloat16.
        config: Optional config dict (no tunables).
    """

    SUPPORTED_DTYPES = (torch.float32, torch.float16, torch.bfloat16)

    def __init__(
        self,
        M: int,
        N: int,
        eps: float,
        dtype: torch.dtype,
        config: Optional[dict] = None,
    ):
        super().__init__()
        check_dtype(self, dtype, self.SUPPORTED_DTYPES)
        self.M = M
        self.N = N
        self.eps = eps
        self.dtype = dtype
        self.init_config(config)

    def forward(
        self,
        x: torch.Tensor,
        residual: torch.Tensor,
        weight: torch.Tensor,
        bias: torch.Tensor,
    ) -> list[torch.Tensor]:
        """Return ``[y, residual_out]`` shaped like ``x``."""
        original_shape = x.shape
        rows = x.contiguous().reshape(-1, self.N)
        residual = residual.contiguous().reshape(-1, self.N)
        weight = weight.contiguous().reshape(self.N)
        bias = bias.contiguous().reshape(self.N)
        if weight.dtype != bias.dtype:
            raise ValueError(f"weight.dtype {weight.dtype} != bias.dtype {bias.dtype}")
        y = torch.empty_like(rows)
        residual_out = torch.empty_like(rows)
        _native.launch(
            "tileops_fused_add_layer_norm_fwd",
            rows.device,
            _native.ptr(rows),
            _native.ptr(residual),
            _native.ptr(weight),
            _native.ptr(bias),
            _native.ptr(y),
            _native.ptr(residual_out),
            rows.shape[0],
            self.N,
            float(self.eps),
            _native.dtype_code(self.dtype),
            _native.dtype_code(weight.dtype),
        )
        return [y.reshape(original_shape), residual_out.reshape(original_shape)]
