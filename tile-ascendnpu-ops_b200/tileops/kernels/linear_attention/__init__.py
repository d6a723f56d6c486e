from tileops.kernels.linear_attention.gdn_prefill import GDNPrefillFwdKernel

__all__ = ["GDNPrefillFwdKernel"]
