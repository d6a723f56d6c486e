"""GeluTanhAndMulFwdOp -- fused gated tanh GELU, y = gelu_tanh(x[:, :N]) * x[:, N:].

Same API as the reference op (ops/elementwise/gelu_tanh_and_mul.py:43-126):
``GeluTanhAndMulFwdOp(M, N, dtype, *, kernel_map=None)``.
"""

from tileops.kernels.elementwise.gelu_tanh_and_mul import GeluTanhAndMulFwdKernel
from tileops.ops.elementwise._gated import GatedFwdOp

__all__ = ["GeluTanhAndMulFwdOp"]


class GeluTanhAndMulFwdOp(GatedFwdOp):
    """``torch.nn.functional.gelu(gate, approximate="tanh") * value``.

    Args:
        M: Number of rows of ``x`` (and of the output).
        N: Output width; ``x`` has ``2 * N`` columns.
        dtype: float16, bfloat16 or float32.
        kernel_map: Optional kernel dispatch override.
    """

    _op_name = "gelu_tanh_and_mul"
    kernel_cls = GeluTanhAndMulFwdKernel
    # Manifest "10 * M * N".
    FLOPS_PER_OUTPUT = 10
