from tileops.ops.linear_attention.gated_delta_net_prefill import GatedDeltaNetPrefillFwdOp

__all__ = ["GatedDeltaNetPrefillFwdOp"]
