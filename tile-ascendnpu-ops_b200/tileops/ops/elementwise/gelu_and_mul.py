"""GeluAndMulFwdOp -- fused gated exact GELU, y = gelu(x[:, :N]) * x[:, N:].

Same API as the reference op (ops/elementwise/gelu_and_mul.py:42-125):
``GeluAndMulFwdOp(M, N, dtype, *, kernel_map=None)``.
"""

from tileops.kernels.elementwise.gelu_and_mul import GeluAndMulFwdKernel
from tileops.ops.elementwise._gated import GatedFwdOp

__all__ = ["GeluAndMulFwdOp"]


class GeluAndMulFwdOp(GatedFwdOp):
    """``torch.nn.functional.gelu(gate, approximate="none") * value``.

    Args:
        M: Number of rows of ``x`` (and of the output).
        N: Output width; ``x`` has ``2 * N`` columns.
        dtype: float16, bfloat16 or float32.
        kernel_map: Optional kernel dispatch override.
    """

    _op_name = "gelu_and_mul"
    kernel_cls = GeluAndMulFwdKernel
    # Manifest "6 * M * N": div, erf, add, mul-by-half, mul-by-gate, mul-by-value.
    FLOPS_PER_OUTPUT = 6
