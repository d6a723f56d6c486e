from tileops.ops.convolution import CausalDepthwiseConv1dFwdOp, Conv1dBiasFwdOp, Conv1dFwdOp
from tileops.ops.op_base import Op

__all__ = ["CausalDepthwiseConv1dFwdOp", "Conv1dBiasFwdOp", "Conv1dFwdOp", "Op"]
