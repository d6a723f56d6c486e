from tileops.kernels.linear_attention.gdn_prefill import GDNPrefillFwdKernel
from tileops.kernels.linear_attention.gla_decode import GLADecodeKernel

__all__ = ["GDNPrefillFwdKernel", "GLADecodeKernel"]
