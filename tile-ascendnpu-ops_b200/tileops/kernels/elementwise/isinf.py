"""IsinfFwdKernel: y = isinf(x) as torch.bool, exact.

Replaces the reference kernel class at kernels/elementwise/isinf/isinf.py:83
(TileLang isinf_fwd_kernel) with the native entry point tileops_isinf_fwd.
"""

from tileops.kernels.elementwise._unary import FLOAT_DTYPES, UnaryNativeKernel

__all__ = ["IsinfFwdKernel"]


class IsinfFwdKernel(UnaryNativeKernel):
    """y = isinf(x) as torch.bool, exact.

    Args:
        N_total: Total number of elements (flattened input).
        dtype: Input dtype (float16, bfloat16 or float32).
        config: Optional config dict (no tunables).
    """

    SUPPORTED_DTYPES = FLOAT_DTYPES
    entry_point = "tileops_isinf_fwd"
    bool_output = True
