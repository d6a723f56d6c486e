from tileops.ops.linear_attention.gla_decode import GLADecodeOp
from tileops.ops.linear_attention.gated_delta_net_prefill import (
    GatedDeltaNetPrefillFwdOp,
    chunk_gated_delta_rule,
)

__all__ = ["GLADecodeOp", "GatedDeltaNetPrefillFwdOp", "chunk_gated_delta_rule"]
