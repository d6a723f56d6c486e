from tileops.kernels.attention.multi_head_attention import GQAPrefillFwdKernel

__all__ = ["GQAPrefillFwdKernel"]
