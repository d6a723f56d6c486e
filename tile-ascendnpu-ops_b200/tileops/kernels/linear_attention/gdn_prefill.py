"""GDNPrefillFwdKernel: gated delta rule, chunked prefill.

Native entry points ``tileops_gdn_prefill_fwd`` and, for packed
variable-length input (``cu_seqlens``), ``tileops_gdn_prefill_varlen_fwd``.
Two kernels: a chunk-parallel prepare kernel computing the WY factors of every
64-token chunk on tensor cores, then a scan over the chunks of each (sequence,
head, 64-column slice of the value dimension), the state in TMEM (tcgen05,
dk = 128) or in fp32 registers (dk = 64).  The reference has no kernel for
this op; its probe kernel is examples/gdn_prefill/probe/gdn_prefill_probe.py:83
and the semantics are its sequential golden at :60-77.

The scratch workspace (per-chunk WY factors) is allocated here through the
torch caching allocator, sized by ``tileops_gdn_workspace_bytes`` /
``tileops_gdn_varlen_workspace_bytes``.
"""

from __future__ import annotations

from typing import Optional

import torch

from tileops import _native
from tileops.kernels.kernel_base import Kernel, check_dtype

__all__ = ["GDNPrefillFwdKernel"]


class GDNPrefillFwdKernel(Kernel):
    """Chunked gated-delta-rule prefill.

    Args:
        batch, seq_len, heads, dim_k, dim_v: problem shape (dim_k, dim_v in {64, 128}).
        chunk_size: 64 (the only supported chunk length).
        scale: Output scale (default ``dim_k ** -0.5``).
        dtype: torch.bfloat16.
        config: Optional config dict (no tunables).
    """

    SUPPORTED_DTYPES = (torch.bfloat16,)
    SUPPORTED_DIMS = (64, 128)

    def __init__(self, batch: int, seq_len: int, heads: int, dim_k: int, dim_v: int,
                 chunk_size: int = 64, scale: Optional[float] = None,
                 dtype: torch.dtype = torch.bfloat16, config: Optional[dict] = None):
        super().__init__()
        check_dtype(self, dtype, self.SUPPORTED_DTYPES)
        if dim_k not in self.SUPPORTED_DIMS or dim_v not in self.SUPPORTED_DIMS:
            raise ValueError(f"{type(self).__name__} supports dim_k, dim_v in "
                             f"{self.SUPPORTED_DIMS}, got ({dim_k}, {dim_v})")
        if chunk_size != 64:
            raise ValueError(f"{type(self).__name__} supports chunk_size 64, got {chunk_size}")
        self.batch, self.seq_len, self.heads = batch, seq_len, heads
        self.dim_k, self.dim_v, self.chunk_size = dim_k, dim_v, chunk_size
        self.scale = dim_k**-0.5 if scale is None else float(scale)
        self.dtype = dtype
        self.init_config(config)

    def workspace_bytes(self) -> int:
        n = _native.lib().tileops_gdn_workspace_bytes(self.batch, self.seq_len, self.heads,
                                                      self.dim_k, self.dim_v)
        if n < 0:
            raise ValueError("unsupported GDN shape")
        return int(n)

    def varlen_workspace_bytes(self, num_seqs: int) -> int:
        n = _native.lib().tileops_gdn_varlen_workspace_bytes(
            self.batch * self.seq_len, num_seqs, self.heads, self.dim_k, self.dim_v)
        if n < 0:
            raise ValueError("unsupported GDN shape")
        return int(n)

    def forward(self, q, k, v, g, beta, initial_state=None, output_final_state: bool = True,
                cu_seqlens=None, use_qk_l2norm_in_kernel: bool = False):
        q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
        g = g.contiguous().float()
        beta = beta.contiguous().float()
        if initial_state is not None:
            initial_state = initial_state.contiguous().float()
        o = torch.empty((self.batch, self.seq_len, self.heads, self.dim_v), dtype=self.dtype,
                        device=q.device)
        # One state per sequence: the batch rows, or the packed sequences.
        nseq = self.batch if cu_seqlens is None else cu_seqlens.numel() - 1
        final = (torch.empty((nseq, self.heads, self.dim_k, self.dim_v),
                             dtype=torch.float32, device=q.device)
                 if output_final_state else None)
        if cu_seqlens is None and not use_qk_l2norm_in_kernel:
            ws = torch.empty(max(self.workspace_bytes(), 16), dtype=torch.uint8,
                             device=q.device)
            _native.launch(
                "tileops_gdn_prefill_fwd", q.device,
                _native.ptr(q), _native.ptr(k), _native.ptr(v), _native.ptr(g),
                _native.ptr(beta), _native.ptr(initial_state), _native.ptr(o),
                _native.ptr(final), _native.ptr(ws),
                self.batch, self.seq_len, self.heads, self.dim_k, self.dim_v, self.chunk_size,
                float(self.scale), _native.dtype_code(self.dtype),
            )
            return o, final
        # The general entry: packed sequences (cu_seqlens) and / or the fused
        # q / k L2 norm; without cu_seqlens it runs `batch` sequences of seq_len.
        cu = (None if cu_seqlens is None
              else cu_seqlens.to(device=q.device, dtype=torch.int32).contiguous())
        ws = torch.empty(max(self.varlen_workspace_bytes(nseq), 16), dtype=torch.uint8,
                         device=q.device)
        flags = _native.GDN_QK_L2NORM if use_qk_l2norm_in_kernel else 0
        _native.launch(
            "tileops_gdn_prefill_varlen_fwd", q.device,
            _native.ptr(q), _native.ptr(k), _native.ptr(v), _native.ptr(g), _native.ptr(beta),
            _native.ptr(cu), nseq, _native.ptr(initial_state), _native.ptr(o),
            _native.ptr(final), _native.ptr(ws),
            self.batch * self.seq_len, self.heads, self.dim_k, self.dim_v, self.chunk_size,
            float(self.scale), flags, _native.dtype_code(self.dtype),
        )
        return o, final
