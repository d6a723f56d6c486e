"""GQAPrefillFwdKernel: flash-style attention forward on tcgen05 / TMEM.

Replaces kernels/attention/multi_head_attention/multi_head_attention.py:132-284
and its TileLang ``_gqa_prefill_fwd_kernel`` with the native entry point
``tileops_mha_fwd``.  BSHD layout: q ``(B, Sq, H, D)``, k / v
``(B, Skv, Hkv, D)``; returns ``(o, lse)`` with ``o`` shaped like q and
``lse`` ``(B, H, Sq)`` float32 in the log2 domain (``logsumexp / ln 2``).
Causal masking is right-aligned.

As in the reference, the call goes through a ``torch.library`` custom op
(``tileops::gqa_prefill_fwd``, reference ``npub::gqa_prefill_fwd_wrapped_kernel``
at :77-124) with a fake implementation, so the op composes with
``torch.compile`` tracing.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch

from tileops import _native
from tileops.kernels.kernel_base import Kernel, check_dtype

__all__ = ["GQAPrefillFwdKernel"]


@torch.library.custom_op("tileops::gqa_prefill_fwd", mutates_args=())
def _gqa_prefill_fwd(
    batch: int,
    heads: int,
    heads_kv: int,
    seq_len_q: int,
    seq_len_kv: int,
    dim: int,
    is_causal: bool,
    sm_scale: float,
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
) -> Tuple[torch.Tensor, torch.Tensor]:
    q = q.contiguous()
    k = k.contiguous()
    v = v.contiguous()
    o = torch.empty_like(q)
    lse = torch.empty((batch, heads, seq_len_q), dtype=torch.float32, device=q.device)
    _native.launch(
        "tileops_mha_fwd",
        q.device,
        _native.ptr(q),
        _native.ptr(k),
        _native.ptr(v),
        _native.ptr(o),
        _native.ptr(lse),
        batch,
        heads,
        heads_kv,
        seq_len_q,
        seq_len_kv,
        dim,
        int(is_causal),
        float(sm_scale),
        _native.dtype_code(q.dtype),
    )
    return o, lse


@_gqa_prefill_fwd.register_fake
def _(batch, heads, heads_kv, seq_len_q, seq_len_kv, dim, is_causal, sm_scale, q, k, v):
    return torch.empty_like(q), q.new_empty([batch, heads, seq_len_q], dtype=torch.float32)


class GQAPrefillFwdKernel(Kernel):
    """GQA / MHA prefill forward (BSHD), online softmax on tcgen05 tensor cores.

    Args:
        batch, heads, heads_kv, seq_len_q, seq_len_kv, dim: problem shape
            (``heads % heads_kv == 0``; causal needs ``seq_len_q <= seq_len_kv``).
        is_causal: Apply the right-aligned causal mask.
        dtype: float16 or bfloat16.
        sm_scale: Softmax scale (default ``dim ** -0.5``).
        softcap: Score softcap; only ``0.0`` (disabled) is implemented.
        config: Optional config dict (no tunables).
    """

    SUPPORTED_DTYPES = (torch.float16, torch.bfloat16)

    def __init__(
        self,
        batch: int,
        heads: int,
        heads_kv: int,
        seq_len_q: int,
        seq_len_kv: int,
        dim: int,
        is_causal: bool,
        dtype: torch.dtype,
        sm_scale: Optional[float] = None,
        softcap: float = 0.0,
        config: Optional[dict] = None,
    ) -> None:
        super().__init__()
        check_dtype(self, dtype, self.SUPPORTED_DTYPES)
        if heads % heads_kv != 0:
            raise ValueError("heads must be divisible by heads_kv")
        if is_causal and seq_len_q > seq_len_kv:
            raise ValueError("causal prefill requires seq_len_q <= seq_len_kv")
        if softcap != 0.0:
            raise ValueError("GQAPrefillFwdKernel: softcap > 0 is not implemented")
        self.batch = batch
        self.heads = heads
        self.heads_kv = heads_kv
        self.seq_len_q = seq_len_q
        self.seq_len_kv = seq_len_kv
        self.dim = dim
        self.is_causal = is_causal
        self.dtype = dtype
        self.sm_scale = dim**-0.5 if sm_scale is None else sm_scale
        self.softcap = softcap
        self.init_config(config)

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor):
        """Return ``(o, lse)`` for BSHD q / k / v."""
        expect_q = (self.batch, self.seq_len_q, self.heads, self.dim)
        expect_kv = (self.batch, self.seq_len_kv, self.heads_kv, self.dim)
        for name, t, shape in (("q", q, expect_q), ("k", k, expect_kv), ("v", v, expect_kv)):
            if tuple(t.shape) != shape:
                raise ValueError(f"Expected {name}.shape {shape}, got {tuple(t.shape)}")
            if t.dtype != self.dtype:
                raise ValueError(f"Expected {name}.dtype {self.dtype}, got {t.dtype}")
        return _gqa_prefill_fwd(
            self.batch, self.heads, self.heads_kv, self.seq_len_q, self.seq_len_kv, self.dim,
            self.is_causal, self.sm_scale, q, k, v,
        )
