"""CPU restatements of the reference's ref programs (test infrastructure only).

Paths are relative to the reference checkout; ``TO/`` is
``examples/TileOPs/``.  Every function takes CPU tensors (device tensors are
copied to the CPU) and returns CPU tensors.  Floating-point ops compute in
fp32 and round once to the input dtype, as the reference programs do;
integer / predicate ops are exact (numpy).
"""

from __future__ import annotations

import math
from typing import Optional

import numpy as np
import torch
import torch.nn.functional as F


def _cpu(t: Optional[torch.Tensor]) -> Optional[torch.Tensor]:
    return None if t is None else t.detach().cpu()


# ---------------------------------------------------------------- unary ops
def hardswish(x: torch.Tensor) -> torch.Tensor:
    """``F.hardswish(x.float()).to(x.dtype)`` -- TO/tests/ops/test_hardswish.py:38-39."""
    x = _cpu(x)
    return F.hardswish(x.float()).to(x.dtype)


def hardsigmoid(x: torch.Tensor) -> torch.Tensor:
    """``F.hardsigmoid(x.float()).to(x.dtype)`` -- TO/tests/ops/test_hardsigmoid.py:38-39."""
    x = _cpu(x)
    return F.hardsigmoid(x.float()).to(x.dtype)


def clamp_scalar(x: torch.Tensor, min_val=None, max_val=None) -> torch.Tensor:
    """``torch.clamp(x.float(), min, max).to(x.dtype)`` -- TO/tests/ops/test_clamp_scalar.py:56-57."""
    x = _cpu(x)
    return torch.clamp(x.float(), min_val, max_val).to(x.dtype)


def clamp_min(x: torch.Tensor, min_val) -> torch.Tensor:
    """``torch.clamp_min(x.float(), min).to(x.dtype)`` -- TO/tests/ops/test_clamp_min.py:48-49."""
    x = _cpu(x)
    return torch.clamp_min(x.float(), min_val).to(x.dtype)


def _as_f32_numpy(x: torch.Tensor) -> np.ndarray:
    return _cpu(x).float().numpy()


def isnan(x: torch.Tensor) -> torch.Tensor:
    """``torch.isnan(x.float())`` -- TO/tests/ops/test_isnan.py:53-58 (numpy, exact)."""
    return torch.from_numpy(np.isnan(_as_f32_numpy(x)))


def isinf(x: torch.Tensor) -> torch.Tensor:
    """``torch.isinf(x.float())`` -- TO/tests/ops/test_isinf.py:54-59 (numpy, exact)."""
    return torch.from_numpy(np.isinf(_as_f32_numpy(x)))


def isfinite(x: torch.Tensor) -> torch.Tensor:
    """``torch.isfinite(x.float())`` -- TO/tests/ops/test_isfinite.py:55-60 (numpy, exact)."""
    return torch.from_numpy(np.isfinite(_as_f32_numpy(x)))


def bitwise_not(x: torch.Tensor) -> torch.Tensor:
    """``torch.bitwise_not(x)`` -- TO/tests/ops/test_bitwise_not.py:53-54 (numpy, exact).

    Integers: two's-complement ``~x``; bool: logical not.
    """
    a = _cpu(x).numpy()
    out = np.logical_not(a) if a.dtype == np.bool_ else np.invert(a)
    return torch.from_numpy(np.ascontiguousarray(out))


# ---------------------------------------------------------------- gated ops
def gelu_and_mul(x: torch.Tensor) -> torch.Tensor:
    """Explicit-erf GELU times value in fp32 -- TO/tests/ops/test_gelu_and_mul.py:63-76.

    ``gelu = 0.5 * g * (1 + erf(g * sqrt(0.5)))``; ``y = (gelu * v).to(dtype)``.
    """
    x = _cpu(x)
    half = x.shape[-1] // 2
    xf = x.float()
    g, v = xf[..., :half], xf[..., half:]
    gelu = 0.5 * g * (1.0 + torch.erf(g * (0.5**0.5)))
    return (gelu * v).to(x.dtype)


def gelu_tanh_and_mul(x: torch.Tensor) -> torch.Tensor:
    """Explicit tanh-GELU times value in fp32 -- TO/tests/ops/test_gelu_tanh_and_mul.py:64-86."""
    x = _cpu(x)
    half = x.shape[-1] // 2
    xf = x.float()
    g, v = xf[..., :half], xf[..., half:]
    inner = math.sqrt(2.0 / math.pi) * (g + 0.044715 * g**3)
    gelu = 0.5 * g * (1.0 + torch.tanh(inner))
    return (gelu * v).to(x.dtype)


# ------------------------------------------------------------------- norm
def fused_add_layer_norm(x, residual, weight, bias, eps: float = 1e-5):
    """Residual add (rounded) then LayerNorm -- TO/tests/ops/test_fused_add_layer_norm.py:55-72.

    ``added = (x.float() + residual.float()).to(dtype)``;
    ``y = F.layer_norm(added.float(), (N,), w.float(), b.float(), eps).to(dtype)``.
    Returns ``(y, added)``.
    """
    x, residual, weight, bias = map(_cpu, (x, residual, weight, bias))
    n = x.shape[-1]
    added = (x.float() + residual.float()).to(x.dtype)
    y = F.layer_norm(added.float(), (n,), weight.float(), bias.float(), eps).to(x.dtype)
    return y, added


# ------------------------------------------------------------ convolution
def conv1d(x, weight, bias=None, stride=1, padding=0, dilation=1, groups=1):
    """``F.conv1d`` in fp32 then one rounding -- TO/tileops/workloads/convolution.py:293-307.

    Depthwise golden: TO/tileops/kernels/convolution/conv1d/conv1d_kernel/_conv1d_direct_kernel.py:134-158.
    """
    x, weight, bias = map(_cpu, (x, weight, bias))
    out = F.conv1d(x.float(), weight.float(), None if bias is None else bias.float(),
                   stride=stride, padding=padding, dilation=dilation, groups=groups)
    return out.to(x.dtype).contiguous()


def causal_depthwise_conv1d(x, weight, bias=None, activation: Optional[str] = None):
    """Causal depthwise conv: ``F.conv1d(x, w, b, padding=K-1, groups=C)[..., :L]`` (+ SiLU) in fp32.

    The causal form is this build's extension (the reference API pads both
    sides); it is the depthwise golden above with left padding only.
    ``weight`` is ``(C, K)`` or ``(C, 1, K)``.
    """
    x, weight, bias = map(_cpu, (x, weight, bias))
    c, length = x.shape[1], x.shape[2]
    w = weight.reshape(c, 1, -1).float()
    k = w.shape[-1]
    out = F.conv1d(x.float(), w, None if bias is None else bias.float(), padding=k - 1,
                   groups=c)[..., :length]
    if activation == "silu":
        out = F.silu(out)
    return out.to(x.dtype).contiguous()


# --------------------------------------------------------------- attention
def mha_sdpa(q, k, v, is_causal: bool) -> torch.Tensor:
    """Output reference of the MHA test: SDPA on BHSD in the input dtype.

    TO/tests/ops/test_multi_head_attention.py:32-44 (no upcast: torch's CPU
    SDPA computes in the input dtype).
    """
    q, k, v = map(_cpu, (q, k, v))
    out = F.scaled_dot_product_attention(
        q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), is_causal=is_causal
    )
    return out.transpose(1, 2).contiguous()


def gqa_prefill_fwd(q, k, v, is_causal: bool, sm_scale: Optional[float] = None):
    """Materialised-softmax attention with a log2-domain LSE.

    Restates golden_gqa_prefill_fwd,
    TO/tileops/kernels/attention/multi_head_attention/multi_head_attention_kernel/perf_opt/_gqa_prefill_fwd_kernel.py:151-194:
    per (b, h) fp32 scores ``scale * q k^T``, right-aligned causal mask,
    ``lse = logsumexp(scores) / ln 2``, ``p = softmax(scores)`` quantised to
    the input dtype before ``p @ v``.  q ``(B, Sq, H, D)``, k / v
    ``(B, Skv, Hkv, D)``.  Returns ``(o, lse)``.
    """
    q, k, v = map(_cpu, (q, k, v))
    batch, sq, heads, dim = q.shape
    skv, heads_kv = k.shape[1], k.shape[2]
    scale = dim**-0.5 if sm_scale is None else sm_scale
    qf = q.transpose(1, 2).float()
    kf = k.transpose(1, 2).float()
    vf = v.transpose(1, 2).float()
    if is_causal:
        valid = (torch.arange(sq)[:, None] + (skv - sq)) >= torch.arange(skv)[None, :]
    o = torch.empty(batch, sq, heads, dim, dtype=q.dtype)
    lse = torch.empty(batch, heads, sq, dtype=torch.float32)
    group = heads // heads_kv
    for b in range(batch):
        for h in range(heads):
            hk = h // group
            s = (qf[b, h] @ kf[b, hk].transpose(-2, -1)) * scale
            if is_causal:
                s = s.masked_fill(~valid, float("-inf"))
            lse[b, h] = torch.logsumexp(s, dim=-1) / math.log(2.0)
            p = torch.softmax(s, dim=-1)
            o[b, :, h, :] = (p.to(q.dtype) @ vf[b, hk].to(q.dtype)).to(q.dtype)
    return o, lse


# ------------------------------------------------------ gated delta net
def gdn_sequential(q, k, v, g, beta, state0, scale: float):
    """Token-by-token gated delta rule in fp32.

    Restates golden_gdn_sequential, examples/gdn_prefill/probe/gdn_prefill_probe.py:60-77
    (layout BHTD there): for every t,
    ``S <- S * exp(g_t)``; ``S <- S + k_t (x) beta_t (v_t - k_t^T S)``;
    ``o_t = scale * q_t^T S``.
    q, k ``(B, H, T, Dk)``; v ``(B, H, T, Dv)``; g, beta ``(B, H, T)``;
    state0 ``(B, H, Dk, Dv)``.  Returns ``(o (B, H, T, Dv) fp32, S fp32)``.
    """
    q, k, v, g, beta, state0 = map(_cpu, (q, k, v, g, beta, state0))
    batch, heads, t_len, _ = q.shape
    dv = v.shape[-1]
    qf, kf, vf = q.float(), k.float(), v.float()
    gf, bf = g.float(), beta.float()
    s = state0.float().clone()
    o = torch.zeros(batch, heads, t_len, dv)
    for t in range(t_len):
        s = s * torch.exp(gf[:, :, t])[:, :, None, None]
        pred = torch.einsum("bhd,bhdv->bhv", kf[:, :, t], s)
        err = bf[:, :, t][:, :, None] * (vf[:, :, t] - pred)
        s = s + kf[:, :, t][:, :, :, None] * err[:, :, None, :]
        o[:, :, t] = scale * torch.einsum("bhd,bhdv->bhv", qf[:, :, t], s)
    return o, s


def l2norm_rows(x, eps: float = 1e-6):
    """``x / sqrt(sum(x^2) + eps)`` over the last dim in fp32, cast back to x's
    dtype: the q / k normalisation fla applies for use_qk_l2norm_in_kernel
    (its l2norm forward, eps 1e-6)."""
    xf = _cpu(x).float()
    return (xf / torch.sqrt((xf * xf).sum(-1, keepdim=True) + eps)).to(x.dtype)


def gdn_prefill_bthd(q, k, v, g, beta, scale: Optional[float] = None, initial_state=None,
                     qk_l2norm: bool = False):
    """The GDN golden on the op's BTHD layout.

    q, k ``(B, T, H, Dk)``, v ``(B, T, H, Dv)``, g / beta ``(B, T, H)``,
    initial_state ``(B, H, Dk, Dv)`` or None (zeros); ``qk_l2norm`` first
    normalises q and k per token and head (``l2norm_rows``).  Returns
    ``(o (B, T, H, Dv) in v's dtype, final_state (B, H, Dk, Dv) fp32)``.
    """
    q, k, v, g, beta = map(_cpu, (q, k, v, g, beta))
    if qk_l2norm:
        q, k = l2norm_rows(q), l2norm_rows(k)
    batch, _, heads, dk = q.shape
    dv = v.shape[-1]
    scale = dk**-0.5 if scale is None else scale
    s0 = torch.zeros(batch, heads, dk, dv) if initial_state is None else _cpu(initial_state)
    o, s = gdn_sequential(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                          g.transpose(1, 2), beta.transpose(1, 2), s0, scale)
    return o.transpose(1, 2).contiguous().to(v.dtype), s


def gdn_prefill_varlen(q, k, v, g, beta, cu_seqlens, scale: Optional[float] = None,
                       initial_state=None, qk_l2norm: bool = False):
    """The GDN golden on packed variable-length input (fla's ``cu_seqlens``).

    q, k ``(1, T, H, Dk)``, v ``(1, T, H, Dv)``, g / beta ``(1, T, H)`` hold N
    sequences, sequence n being tokens ``cu_seqlens[n]:cu_seqlens[n + 1]``;
    initial_state ``(N, H, Dk, Dv)`` or None.  Every sequence runs the
    sequential recurrence (golden_gdn_sequential,
    examples/gdn_prefill/probe/gdn_prefill_probe.py:60-77) from its own initial
    state.  Returns ``(o (1, T, H, Dv), final_state (N, H, Dk, Dv) fp32)``.
    """
    q, k, v, g, beta = map(_cpu, (q, k, v, g, beta))
    cu = [int(x) for x in _cpu(cu_seqlens).tolist()]
    heads, dk, dv = q.shape[2], q.shape[3], v.shape[3]
    o = torch.zeros(v.shape, dtype=v.dtype)
    finals = []
    for n in range(len(cu) - 1):
        a, b = cu[n], cu[n + 1]
        h0 = None if initial_state is None else _cpu(initial_state)[n:n + 1]
        if b == a:
            finals.append(torch.zeros(1, heads, dk, dv) if h0 is None else h0.float().clone())
            continue
        o_n, s_n = gdn_prefill_bthd(q[:, a:b], k[:, a:b], v[:, a:b], g[:, a:b], beta[:, a:b],
                                    scale, h0, qk_l2norm)
        o[:, a:b] = o_n
        finals.append(s_n)
    final = torch.cat(finals, 0) if finals else torch.zeros(0, heads, dk, dv)
    return o, final


# ------------------------------------------------------ GLA decode
def gla_decode(q, k, v, gk, state, scale: float):
    """One gated-linear-attention decode step in fp32.

    Restates golden_gla_decode,
    examples/TileOPs/tileops/kernels/linear_attention/gla_decode/gla_decode_kernel/
    _gla_decode_kernel.py:211-218 (layout BHD): new_state = exp(gk)[..., None]
    * state + k (x) v; o = scale * q^T new_state.  Returns ``(o, new_state)``
    in fp32.
    """
    qf, kf, vf, gf, sf = (_cpu(t).float() for t in (q, k, v, gk, state))
    new_state = sf * torch.exp(gf)[..., None] + kf[..., :, None] * vf[..., None, :]
    o = scale * torch.einsum("bhk,bhkv->bhv", qf, new_state)
    return o, new_state


# ------------------------------------------------------ Mamba-2 SSD chunk scan
def ssd_chunk_scan(x, cb, dA_cumsum, C, prev_states, dt, n_groups: int):
    """Fused SSD chunk output in fp32.

    Restates golden_ssd_chunk_scan_fwd,
    examples/TileOPs/tileops/kernels/mamba/ssd_chunk_scan/ssd_chunk_scan_kernel/perf_opt/
    _ssd_chunk_scan_fwd_kernel.py:123-178:
    out[l, p] = exp(dA[l]) sum_n C[l, n] prev[p, n]
              + sum_{s <= l} cb[l, s] exp(dA[l] - dA[s]) dt[s] x[s, p],
    per batch, chunk and head (group h // (H // G)).  Layouts: x (B, S, H, P),
    cb (B, NC, G, L, L), dA_cumsum (B, H, NC, L), C (B, S, G, N), prev_states
    (B, NC, H, P, N), dt (B, H, NC, L); returns (B, S, H, P) fp32.
    """
    x, cb, dA_cumsum, C, prev_states, dt = map(_cpu, (x, cb, dA_cumsum, C, prev_states, dt))
    b, seq, h, p = x.shape
    nc, L = dA_cumsum.shape[2], dA_cumsum.shape[3]
    n = C.shape[-1]
    head_group = torch.arange(h) // (h // n_groups)
    Ch = C.float().reshape(b, nc, L, n_groups, n)[:, :, :, head_group, :]   # B NC L H N
    dA = dA_cumsum.float()                                                  # B H NC L
    hist = torch.einsum("bclhn,bchpn->bclhp", Ch, prev_states.float())
    hist = hist * torch.exp(dA.permute(0, 2, 3, 1)).unsqueeze(-1)
    causal = torch.tril(torch.ones(L, L, dtype=torch.bool))
    decay = torch.exp(dA.unsqueeze(-1) - dA.unsqueeze(-2)).masked_fill(~causal, 0.0)
    weight = (cb.float()[:, :, head_group] * decay.permute(0, 2, 1, 3, 4)
              * dt.float().permute(0, 2, 1, 3).unsqueeze(-2))                  # B NC H L L
    intra = torch.einsum("bchls,bcshp->bclhp", weight, x.float().reshape(b, nc, L, h, p))
    return (hist + intra).reshape(b, seq, h, p)
