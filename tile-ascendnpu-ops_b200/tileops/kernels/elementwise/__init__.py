from tileops.kernels.elementwise.bitwise_not import BitwiseNotFwdKernel
from tileops.kernels.elementwise.clamp_scalar import ClampScalarFwdKernel
from tileops.kernels.elementwise.gelu_and_mul import GeluAndMulFwdKernel
from tileops.kernels.elementwise.gelu_tanh_and_mul import GeluTanhAndMulFwdKernel
from tileops.kernels.elementwise.hardsigmoid import HardsigmoidFwdKernel
from tileops.kernels.elementwise.hardswish import HardswishFwdKernel
from tileops.kernels.elementwise.isfinite import IsfiniteFwdKernel
from tileops.kernels.elementwise.isinf import IsinfFwdKernel
from tileops.kernels.elementwise.isnan import IsnanFwdKernel

__all__ = [
    "BitwiseNotFwdKernel",
    "ClampScalarFwdKernel",
    "GeluAndMulFwdKernel",
    "GeluTanhAndMulFwdKernel",
    "HardsigmoidFwdKernel",
    "HardswishFwdKernel",
    "IsfiniteFwdKernel",
    "IsinfFwdKernel",
    "IsnanFwdKernel",
]
