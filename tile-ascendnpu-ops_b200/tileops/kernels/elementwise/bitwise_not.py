"""BitwiseNotFwdKernel: y = ~x for integers, logical not for bool.

Replaces kernels/elementwise/bitwise_not/bitwise_not.py:89 (TileLang
bitwise_not_fwd_kernel) with tileops_bitwise_not_fwd, a 16-byte XOR stream.
"""

import torch

from tileops.kernels.elementwise._unary import UnaryNativeKernel

__all__ = ["BitwiseNotFwdKernel"]


class BitwiseNotFwdKernel(UnaryNativeKernel):
    """Bitwise NOT over bool / uint8 / int8 / int16 / int32 / int64.

    Args:
        N_total: Total number of elements (flattened input).
        dtype: bool, uint8, int8, int16, int32 or int64.
        config: Optional config dict (no tunables).
    """

    SUPPORTED_DTYPES = (
        torch.bool,
        torch.uint8,
        torch.int8,
        torch.int16,
        torch.int32,
        torch.int64,
    )
    entry_point = "tileops_bitwise_not_fwd"
