"""IsfiniteFwdKernel: y = isfinite(x) as torch.bool, exact.

Replaces the reference kernel class at kernels/elementwise/isfinite/isfinite.py:82
(TileLang isfinite_fwd_kernel) with the native entry point tileops_isfinite_fwd.
"""

from tileops.kernels.elementwise._unary import FLOAT_DTYPES, UnaryNativeKernel

__all__ = ["IsfiniteFwdKernel"]


class IsfiniteFwdKernel(UnaryNativeKernel):
    """y = isfinite(x) as torch.bool, exact.

    Args:
        N_total: Total number of elements (flattened input).
        dtype: Input dtype (float16, bfloat16 or float32).
        config: Optional config dict (no tunables).
    """

    SUPPORTED_DTYPES = FLOAT_DTYPES
    entry_point = "tileops_isfinite_fwd"
    bool_output = True
