from tileops.ops.norm.fused_add_layer_norm import FusedAddLayerNormFwdOp

__all__ = ["FusedAddLayerNormFwdOp"]
