from tileops.ops.linear_attention.gated_delta_net_prefill import (
    GatedDeltaNetPrefillFwdOp,
    chunk_gated_delta_rule,
)

__all__ = ["GatedDeltaNetPrefillFwdOp", "chunk_gated_delta_rule"]
