from tileops.kernels.norm.fused_add_layer_norm import FusedAddLayerNormKernel

__all__ = ["FusedAddLayerNormKernel"]
