"""SSDChunkScanFwdKernel: Mamba-2 SSD fused chunk output, forward.

Native entry point ``tileops_ssd_chunk_scan_fwd``: one CTA per (batch, chunk,
head, 128-row tile of the chunk), the history term ``C . prev^T`` and the
intra-chunk term ``W . x`` (W = cb * exp(dA_l - dA_s) * dt_s, causal) as two
tcgen05 MMAs with fp32 accumulators in TMEM.  Replaces the reference factory
kernels/mamba/ssd_chunk_scan/ssd_chunk_scan_kernel/perf_opt/_ssd_chunk_scan_fwd_kernel.py:181
behind the same class (kernels/mamba/ssd_chunk_scan/ssd_chunk_scan.py:160-260):
same constructor, ``default_config`` keys (tile sizes of the reference
kernel, kept for interface compatibility; the CUDA kernel's tiles are fixed)
and the fp32 ``(B, S, H, P)`` output.
"""

from __future__ import annotations

from typing import Optional

import torch

from tileops import _native
from tileops.kernels.kernel_base import Kernel, check_dtype

__all__ = ["SSDChunkScanFwdKernel"]


class SSDChunkScanFwdKernel(Kernel):
    """Mamba-2 SSD fused chunk output forward kernel (layouts of mamba_ssm
    ``_chunk_scan_fwd``): x (B, S, H, P), cb (B, C, G, L, L), C (B, S, G, N)
    and dt (B, H, C, L) in ``dtype``; dA_cumsum (B, H, C, L) and prev_states
    (B, C, H, P, N) fp32; out (B, S, H, P) fp32."""

    supported_archs: Optional[list] = [100]
    SUPPORTED_DTYPES = (torch.float16, torch.bfloat16)

    def __init__(self, batch: int, num_chunks: int, chunk_len: int, n_heads: int, d_head: int,
                 d_state: int, n_groups: int, dtype: torch.dtype, config: Optional[dict] = None,
                 device_index: int | None = None) -> None:
        super().__init__()
        check_dtype(self, dtype, self.SUPPORTED_DTYPES)
        if n_heads % n_groups != 0:
            raise ValueError("n_heads must be divisible by n_groups")
        if d_head % 16 != 0 or not 16 <= d_head <= 128:
            raise ValueError(f"{type(self).__name__} supports d_head in 16..128, a multiple of "
                             f"16, got {d_head}")
        if d_state % 8 != 0 or not 8 <= d_state <= 256:
            raise ValueError(f"{type(self).__name__} supports d_state in 8..256, a multiple of "
                             f"8, got {d_state}")
        if not 1 <= chunk_len <= 1024:
            raise ValueError(f"{type(self).__name__} supports chunk_len up to 1024, got "
                             f"{chunk_len}")
        self.batch = batch
        self.num_chunks = num_chunks
        self.chunk_len = chunk_len
        self.n_heads = n_heads
        self.d_head = d_head
        self.d_state = d_state
        self.n_groups = n_groups
        self.dtype = dtype
        self.device_index = device_index
        self.init_config(config)

    @property
    def default_config(self) -> dict:
        return {"block_l": 64, "block_p": 64, "block_n": min(128, self.d_state), "block_s": 64,
                "num_stages": 2}

    def forward(self, x: torch.Tensor, cb: torch.Tensor, dA_cumsum: torch.Tensor,
                C: torch.Tensor, prev_states: torch.Tensor, dt: torch.Tensor) -> torch.Tensor:
        x, cb, C, dt = (t.contiguous() for t in (x, cb, C, dt))
        dA_cumsum = dA_cumsum.contiguous().float()
        prev_states = prev_states.contiguous().float()
        out = torch.empty((self.batch, self.num_chunks * self.chunk_len, self.n_heads,
                           self.d_head), dtype=torch.float32, device=x.device)
        _native.launch(
            "tileops_ssd_chunk_scan_fwd", x.device,
            _native.ptr(x), _native.ptr(cb), _native.ptr(dA_cumsum), _native.ptr(C),
            _native.ptr(prev_states), _native.ptr(dt), _native.ptr(out),
            self.batch, self.num_chunks, self.chunk_len, self.n_heads, self.d_head,
            self.d_state, self.n_groups, _native.dtype_code(self.dtype),
        )
        return out
