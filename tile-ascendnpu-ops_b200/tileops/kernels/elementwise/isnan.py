"""IsnanFwdKernel: y = isnan(x) as torch.bool, exact.

Replaces the reference kernel class at kernels/elementwise/isnan/isnan.py:75
(TileLang isnan_fwd_kernel) with the native entry point tileops_isnan_fwd.
"""

from tileops.kernels.elementwise._unary import FLOAT_DTYPES, UnaryNativeKernel

__all__ = ["IsnanFwdKernel"]


class IsnanFwdKernel(UnaryNativeKernel):
    """y = isnan(x) as torch.bool, exact.

    Args:
        N_total: Total number of elements (flattened input).
        dtype: Input dtype (float16, bfloat16 or float32).
        config: Optional config dict (no tunables).
    """

    SUPPORTED_DTYPES = FLOAT_DTYPES
    entry_point = "tileops_isnan_fwd"
    bool_output = True
