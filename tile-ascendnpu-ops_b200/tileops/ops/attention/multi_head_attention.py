"""MultiHeadAttentionFwdOp -- attention forward, BSHD layout.

Same API as the reference op (ops/attention/multi_head_attention.py:34-120):
``MultiHeadAttentionFwdOp(batch, heads, seq_len, dim, is_causal=True,
dtype=torch.float16, kernel_map=None)``; the kernel key is
``"gqa_prefill_fwd_kernel"`` (MHA is GQA with ``heads_kv == heads``, scale
``dim ** -0.5``, no softcap), ``forward(q, k, v) -> (output, lse)``.
"""

from typing import Dict, Optional

import torch

from tileops.device import get_device_backend
from tileops.kernels.attention.multi_head_attention import GQAPrefillFwdKernel
from tileops.kernels.kernel_base import Kernel
from tileops.ops.op_base import Op

__all__ = ["MultiHeadAttentionFwdOp"]


class MultiHeadAttentionFwdOp(Op):
    """Multi-head attention forward.

    Args:
        batch: Batch size.
        heads: Number of heads.
        seq_len: Sequence length (query and kv).
        dim: Head dimension.
        is_causal: Apply a causal mask.
        dtype: float16 or bfloat16.
        kernel_map: Optional override for kernel dispatch.
    """

    def __init__(
        self,
        batch: int,
        heads: int,
        seq_len: int,
        dim: int,
        is_causal: bool = True,
        dtype: torch.dtype = torch.float16,
        kernel_map: Optional[Dict[str, Kernel]] = None,
    ) -> None:
        self.batch = batch
        self.heads = heads
        self.seq_len = seq_len
        self.dim = dim
        self.is_causal = is_causal
        self.dtype = dtype
        self.dispatch_kernel(kernel_map)
        self.kernel: Kernel = self.kernel_map["gqa_prefill_fwd_kernel"](
            batch, heads, heads, seq_len, seq_len, dim, is_causal, dtype,
            sm_scale=dim**-0.5, softcap=0.0,
        )

    @property
    def default_kernel_map(self) -> Dict[str, Kernel]:
        return {"gqa_prefill_fwd_kernel": GQAPrefillFwdKernel}

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor):
        """Run attention on BSHD q / k / v; returns ``(output, lse)``."""
        backend = get_device_backend()
        for name, t in (("q", q), ("k", k), ("v", v)):
            if not backend.is_device_tensor(t):
                raise ValueError(f"{name} must be a {backend.name} tensor, got device {t.device}")
        return self.kernel(q, k, v)

    def eval_roofline(self) -> tuple[int, int]:
        """``4 * B * H * S^2 * D`` flops (halved when causal); q/k/v read + o written."""
        elem_bytes = self.dtype.itemsize
        flops = 4 * self.batch * self.heads * self.seq_len * self.seq_len * self.dim
        if self.is_causal:
            flops //= 2
        q_elems = self.batch * self.seq_len * self.heads * self.dim
        return int(flops), int(2 * (q_elems + q_elems) * elem_bytes)
