"""GatedDeltaNetPrefillFwdOp -- gated delta rule (Gated DeltaNet) chunked prefill.

The reference names this interface (the migration task lists
``GatedDeltaNetPrefillFwdOp``; baseline op key ``GDNFwdOp``, ref_api
``fla.ops.gated_delta_rule.chunk_gated_delta_rule``) but never delivered it
(examples/gdn_prefill/DESIGN.md); its semantics are the sequential golden
examples/gdn_prefill/probe/gdn_prefill_probe.py:60-77.  This build defines the
API in the style of the other ops:

    GatedDeltaNetPrefillFwdOp(batch, seq_len, heads, dim_k, dim_v, chunk_size=64,
                              scale=None, dtype=torch.bfloat16, kernel_map=None)
    forward(q, k, v, g, beta, initial_state=None, cu_seqlens=None,
            use_qk_l2norm_in_kernel=False) -> (o, final_state)

Layout BTHD (the fla convention): q, k (B, T, H, dk), v (B, T, H, dv) bf16; g
(B, T, H) fp32 per-token log decay (<= 0 for decay); beta (B, T, H) fp32;
initial_state (B, H, dk, dv) fp32 or None (zeros).  Returns o (B, T, H, dv)
bf16 and the final state (B, H, dk, dv) fp32; passing it as the next call's
initial_state continues the sequence (chunked prefill of long contexts).

Variable-length input follows fla's ``cu_seqlens`` convention: batch 1, the N
sequences packed along the token axis, ``cu_seqlens`` an integer device tensor
of N + 1 offsets (0, ..., T); initial_state and the final state are then
(N, H, dk, dv), one per sequence.  ``use_qk_l2norm_in_kernel`` uses
q / sqrt(|q|^2 + 1e-6) and k likewise per token and head (fla's l2norm), fused
into the kernels: q and k are read once, never rewritten.

``chunk_gated_delta_rule`` is the fla-style functional form.
"""

from __future__ import annotations

from typing import Dict, Optional

import torch

from tileops.device import get_device_backend
from tileops.kernels.kernel_base import Kernel
from tileops.kernels.linear_attention import GDNPrefillFwdKernel
from tileops.ops.op_base import Op

__all__ = ["GatedDeltaNetPrefillFwdOp", "chunk_gated_delta_rule"]


class GatedDeltaNetPrefillFwdOp(Op):
    """Chunked gated delta rule prefill.

    Args:
        batch, seq_len, heads: Batch size, tokens, heads.
        dim_k, dim_v: Key / value head dimensions (64 or 128).
        chunk_size: Chunk length of the chunked algorithm (64).
        scale: Output scale, default ``dim_k ** -0.5``.
        dtype: torch.bfloat16.
        kernel_map: Optional override of ``"gdn_prefill"``.
    """

    def __init__(self, batch: int, seq_len: int, heads: int, dim_k: int, dim_v: int,
                 chunk_size: int = 64, scale: Optional[float] = None,
                 dtype: torch.dtype = torch.bfloat16,
                 kernel_map: Optional[Dict[str, Kernel]] = None) -> None:
        self.batch, self.seq_len, self.heads = batch, seq_len, heads
        self.dim_k, self.dim_v, self.chunk_size = dim_k, dim_v, chunk_size
        self.scale = scale
        self.dtype = dtype
        self.dispatch_kernel(kernel_map)
        self.kernel = self.kernel_map["gdn_prefill"](batch, seq_len, heads, dim_k, dim_v,
                                                     chunk_size, scale, dtype)

    @property
    def default_kernel_map(self) -> Dict[str, Kernel]:
        return {"gdn_prefill": GDNPrefillFwdKernel}

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g: torch.Tensor,
                beta: torch.Tensor, initial_state: Optional[torch.Tensor] = None,
                cu_seqlens: Optional[torch.Tensor] = None,
                use_qk_l2norm_in_kernel: bool = False):
        backend = get_device_backend()
        for name, t in (("q", q), ("k", k), ("v", v), ("g", g), ("beta", beta),
                        ("initial_state", initial_state), ("cu_seqlens", cu_seqlens)):
            if t is not None and not backend.is_device_tensor(t):
                raise ValueError(f"{name} must be a {backend.name} tensor, got device {t.device}")
        B, T, H, dk, dv = self.batch, self.seq_len, self.heads, self.dim_k, self.dim_v
        for name, t, shape in (("q", q, (B, T, H, dk)), ("k", k, (B, T, H, dk)),
                               ("v", v, (B, T, H, dv)), ("g", g, (B, T, H)),
                               ("beta", beta, (B, T, H))):
            if tuple(t.shape) != shape:
                raise ValueError(f"Expected {name}.shape {shape}, got {tuple(t.shape)}")
        for name, t in (("q", q), ("k", k), ("v", v)):
            if t.dtype != self.dtype:
                raise ValueError(f"Expected {name}.dtype {self.dtype}, got {t.dtype}")
        nseq = B
        if cu_seqlens is not None:
            if B != 1:
                raise ValueError(f"The batch size is expected to be 1 rather than {B} when "
                                 "using `cu_seqlens`. Please flatten variable-length inputs "
                                 "before processing.")
            if cu_seqlens.dim() != 1 or cu_seqlens.numel() < 1:
                raise ValueError("cu_seqlens must be a 1-D tensor of N + 1 offsets, got shape "
                                 f"{tuple(cu_seqlens.shape)}")
            if cu_seqlens.dtype not in (torch.int32, torch.int64):
                raise ValueError(f"cu_seqlens must be int32 or int64, got {cu_seqlens.dtype}")
            nseq = cu_seqlens.numel() - 1
        if initial_state is not None and tuple(initial_state.shape) != (nseq, H, dk, dv):
            raise ValueError(f"Expected initial_state shape {(nseq, H, dk, dv)}, "
                             f"got {tuple(initial_state.shape)}")
        return self.kernel(q, k, v, g, beta, initial_state, cu_seqlens=cu_seqlens,
                           use_qk_l2norm_in_kernel=use_qk_l2norm_in_kernel)

    def eval_roofline(self) -> tuple[int, int]:
        """Dense matmul flops of the chunked WY form and the bytes moved once.

        Per token and head: 2 C dk (k k^T) + 2 C dk (q k^T) + 3 * 2 dk dv (K S,
        Q S, K^T err) + C dv (triangular apply) + 2 C dv (intra-chunk
        (q k^T) err) with C = chunk_size -- 155,648 at C = 64, dk = dv = 128.
        Bytes: q, k, v, o in the input dtype, g and beta fp32, the fp32
        final state (and the initial state when given is not counted).
        """
        C, dk, dv = self.chunk_size, self.dim_k, self.dim_v
        tokens = self.batch * self.seq_len * self.heads
        flops = tokens * (4 * C * dk + 6 * dk * dv + 3 * C * dv)
        eb = self.dtype.itemsize
        nbytes = (tokens * (2 * dk + 2 * dv) * eb + tokens * 2 * 4
                  + self.batch * self.heads * dk * dv * 4)
        return int(flops), int(nbytes)


def chunk_gated_delta_rule(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g: torch.Tensor,
                           beta: torch.Tensor, scale: Optional[float] = None,
                           initial_state: Optional[torch.Tensor] = None,
                           output_final_state: bool = False,
                           use_qk_l2norm_in_kernel: bool = False,
                           cu_seqlens: Optional[torch.Tensor] = None):
    """fla-style functional form (``fla.ops.gated_delta_rule.chunk_gated_delta_rule``
    argument names and order, BTHD layout, chunk 64).

    Returns ``(o, final_state)``; final_state is None unless output_final_state.
    """
    if q.dim() != 4 or v.dim() != 4:
        raise ValueError(f"Expected q (B, T, H, K) and v (B, T, H, V), got {tuple(q.shape)} "
                         f"and {tuple(v.shape)}")
    batch, seq_len, heads, dim_k = q.shape
    op = GatedDeltaNetPrefillFwdOp(batch, seq_len, heads, dim_k, v.shape[-1], scale=scale,
                                   dtype=q.dtype)
    o, final = op(q, k, v, g, beta, initial_state, cu_seqlens=cu_seqlens,
                  use_qk_l2norm_in_kernel=use_qk_l2norm_in_kernel)
    return o, (final if output_final_state else None)
