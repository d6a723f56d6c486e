from tileops.ops.elementwise.bitwise_not import BitwiseNotFwdOp
from tileops.ops.elementwise.clamp_min import ClampMinFwdOp
from tileops.ops.elementwise.clamp_scalar import ClampScalarFwdOp
from tileops.ops.elementwise.gelu_and_mul import GeluAndMulFwdOp
from tileops.ops.elementwise.gelu_tanh_and_mul import GeluTanhAndMulFwdOp
from tileops.ops.elementwise.hardsigmoid import HardsigmoidFwdOp
from tileops.ops.elementwise.hardswish import HardswishFwdOp
from tileops.ops.elementwise.isfinite import IsfiniteFwdOp
from tileops.ops.elementwise.isinf import IsinfFwdOp
from tileops.ops.elementwise.isnan import IsnanFwdOp

__all__ = [
    "BitwiseNotFwdOp",
    "ClampMinFwdOp",
    "ClampScalarFwdOp",
    "GeluAndMulFwdOp",
    "GeluTanhAndMulFwdOp",
    "HardsigmoidFwdOp",
    "HardswishFwdOp",
    "IsfiniteFwdOp",
    "IsinfFwdOp",
    "IsnanFwdOp",
]
