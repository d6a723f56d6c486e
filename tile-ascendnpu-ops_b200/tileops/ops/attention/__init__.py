from tileops.ops.attention.multi_head_attention import MultiHeadAttentionFwdOp

__all__ = ["MultiHeadAttentionFwdOp"]
