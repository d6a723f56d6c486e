from tileops.kernels.convolution.conv1d import (
    Conv1dKernel,
    Conv1dPointwiseKernel,
    Conv1dUnitStrideKernel,
    DepthwiseConv1dKernel,
    GroupConv1dKernel,
)

__all__ = [
    "Conv1dKernel",
    "Conv1dPointwiseKernel",
    "Conv1dUnitStrideKernel",
    "DepthwiseConv1dKernel",
    "GroupConv1dKernel",
]
