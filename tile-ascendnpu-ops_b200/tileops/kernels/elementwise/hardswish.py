"""HardswishFwdKernel: y = x * clamp(x + 3, 0, 6) / 6 (fp32 opmath, one rounding).

Replaces the reference kernel class at kernels/elementwise/hardswish/hardswish.py:82
(TileLang hardswish_fwd_kernel) with the native entry point tileops_hardswish_fwd.
"""

from tileops.kernels.elementwise._unary import FLOAT_DTYPES, UnaryNativeKernel

__all__ = ["HardswishFwdKernel"]


class HardswishFwdKernel(UnaryNativeKernel):
    """y = x * clamp(x + 3, 0, 6) / 6 (fp32 opmath, one rounding).

    Args:
        N_total: Total number of elements (flattened input).
        dtype: Input dtype (float16, bfloat16 or float32).
        config: Optional config dict (no tunables).
    """

    SUPPORTED_DTYPES = FLOAT_DTYPES
    entry_point = "tileops_hardswish_fwd"
    bool_output = False
