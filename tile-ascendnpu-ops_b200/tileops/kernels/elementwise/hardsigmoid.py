"""HardsigmoidFwdKernel: y = clamp(x + 3, 0, 6) / 6 (fp32 opmath, NaN propagates).

Replaces the reference kernel class at kernels/elementwise/hardsigmoid/hardsigmoid.py:78
(TileLang hardsigmoid_fwd_kernel) with the native entry point tileops_hardsigmoid_fwd.
"""

from tileops.kernels.elementwise._unary import FLOAT_DTYPES, UnaryNativeKernel

__all__ = ["HardsigmoidFwdKernel"]


class HardsigmoidFwdKernel(UnaryNativeKernel):
    """y = clamp(x + 3, 0, 6) / 6 (fp32 opmath, NaN propagates).

    Args:
        N_total: Total number of elements (flattened input).
        dtype: Input dtype (float16, bfloat16 or float32).
        config: Optional config dict (no tunables).
    """

    SUPPORTED_DTYPES = FLOAT_DTYPES
    entry_point = "tileops_hardsigmoid_fwd"
    bool_output = False
