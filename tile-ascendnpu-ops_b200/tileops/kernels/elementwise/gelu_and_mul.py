"""GeluAndMulFwdKernel: y = gelu(gate) * value with the exact erf GELU,
gate = x[:, :N], value = x[:, N:].

Replaces kernels/elementwise/gelu_and_mul/gelu_and_mul.py:71-147 (TileLang
gelu_and_mul_fwd_kernel) with the native entry point tileops_gelu_and_mul_fwd:
one (M, 2N) input, one (M, N) output, fp32 math and one rounding per output
element.
"""

from typing import Optional

import torch

from tileops import _native
from tileops.kernels.elementwise._unary import FLOAT_DTYPES
from tileops.kernels.kernel_base import Kernel, check_dtype

__all__ = ["GeluAndMulFwdKernel"]


class GeluAndMulFwdKernel(Kernel):
    """Fused gated activation kernel.

    Args:
        M: Number of rows of ``x`` (and of the output).
        N: Output width; ``x`` has ``2 * N`` columns.
        dtype: float16, bfloat16 or float32.
        config: Optional config dict (no tunables).
    """

    SUPPORTED_DTYPES = FLOAT_DTYPES

    def __init__(self, M: int, N: int, dtype: torch.dtype, config: Optional[dict] = None):
        super().__init__()
        check_dtype(self, dtype, self.SUPPORTED_DTYPES)
        self.M = int(M)
        self.N = int(N)
        self.dtype = dtype
        self.output_dtype = dtype
        self.init_config(config)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """Map a contiguous ``(M, 2N)`` tensor to ``(M, N)``."""
        x = x.contiguous()
        y = torch.empty((self.M, self.N), dtype=self.dtype, device=x.device)
        _native.launch(
            "tileops_gelu_and_mul_fwd",
            x.device,
            _native.ptr(x),
            _native.ptr(y),
            self.M,
            self.N,
            _native.dtype_code(self.dtype),
        )
        return y
