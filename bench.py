"""Benchmark of the hot path on B200: one JSON line per run.

Headline: FusedAddLayerNormFwdOp on x, residual
(8192, 4096) bf16 ~ N(0, 1) with fp32 weight = 1 + 0.1 N(0,1), bias =
0.1 N(0,1), eps 1e-5.  ``--op`` picks another headline op.  The same line
carries ``per_op``: every other hot-path op at its BASELINE configuration
(plus, at N = 1, the reference-manifest workloads of the ops beyond
BASELINE), each timed with the same protocol and with its own roofline,
end-to-end figure, clock record and CPU baseline.

One GPU (N = 1): a step is one op call over the whole BASELINE problem.
The K timed steps replay a CUDA graph of up to 64 consecutive calls, each
with its own outputs, inputs rotating over buffer sets whose total exceeds
the 126 MB L2 (so no step finds its inputs in L2); CUDA events around every
replay.  ``value`` = algorithmic work (the op's ``eval_roofline``) x K /
that time.

N GPUs (torchrun, one rank per GPU, NCCL): the SAME BASELINE problem is
split across the ranks (rows / batches / (batch, head) pairs; every rank
draws the full problem from the same seed and keeps its slice), and a step
is the op on the rank's shard followed by the reassembly of every output on
every rank (``all_gather_into_tensor`` over NVLink; a local permute when
heads were split).  ``value`` = the problem's work x K / the slowest rank's
time for K such steps: strong scaling.  ``kernel_only`` gives the same
problem timed without the reassembly, ``gather`` its bytes and time,
``weak`` the old per-rank replica figure.

``e2e`` times the public op API from pinned HOST buffers: the problem (or
the rank's shard) is cut into chunks; per chunk, the host-to-device copy,
the op call and the device-to-host copy of its outputs run on three
streams, so copies in both directions overlap the kernels.  ``cpu_baseline``
(rank 0, N = 1) times the reference's own torch CPU program (restated in
``oracle/``) on the full configuration wherever one call fits the time
budget, with all host threads.

``--impl reference`` times that CPU program instead (rank 0 only).

Run: python bench.py [--gpus N] [--steps K] [--warmup W] [--op NAME] [--impl ours|reference]
(N > 1: python -m torch.distributed.run --nproc-per-node N bench.py --gpus N ...)
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from dataclasses import dataclass, field
from pathlib import Path
from typing import Callable, Optional

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "tile-ascendnpu-ops_b200"))
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

L2_BYTES = 126 * 1024 * 1024
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
SEED = 1235


# ----------------------------------------------------------------- sharding
def split_range(n: int, index: int, count: int) -> Optional[slice]:
    """The index-th of ``count`` equal contiguous parts of range(n), or None
    when n does not split evenly (``all_gather_into_tensor`` needs equal
    shards on every rank)."""
    if count < 1 or not 0 <= index < count or n % count:
        return None
    per = n // count
    return slice(index * per, (index + 1) * per)


def shard_axis0(t: torch.Tensor, index: int, count: int) -> Optional[torch.Tensor]:
    s = split_range(t.shape[0], index, count)
    return None if s is None else t[s].contiguous()


def bh_split(batch: int, heads: int, index: int, count: int):
    """(batch slice, head slice) of the index-th of ``count`` equal groups of
    (batch, head) pairs, batch-major: whole batches while ``count`` divides
    the batch, else equal head groups inside each batch."""
    bs = split_range(batch, index, count)
    if bs is not None:
        return bs, slice(0, heads)
    if count % batch:
        return None
    per_b = count // batch
    hs = split_range(heads, index % per_b, per_b)
    if hs is None:
        return None
    b = index // per_b
    return slice(b, b + 1), hs


def head_groups(batch: int, count: int) -> int:
    """Head groups per batch in ``bh_split`` (1 when whole batches are split)."""
    return 1 if batch % count == 0 else count // batch


def unshard_bthd(flat: torch.Tensor, batch: int, seq: int, heads: int, dim: int,
                 count: int) -> torch.Tensor:
    """BTHD tensor from ``count`` gathered ``bh_split`` shards (rank-major)."""
    g = head_groups(batch, count)
    if g == 1:
        return flat.view(batch, seq, heads, dim)
    return (flat.view(batch, g, seq, heads // g, dim).permute(0, 2, 1, 3, 4)
            .reshape(batch, seq, heads, dim))


# ----------------------------------------------------------------- workloads
@dataclass
class Workload:
    """One op at one configuration."""

    name: str
    metric: str
    unit: str  # "GB/s" or "TFLOP/s"
    dtype: str
    config: dict
    make_inputs: Callable[[torch.device, int], tuple]  # the full problem on a device
    build_op: Callable[[tuple], object]  # an op sized for these inputs
    run: Callable[[object, tuple], object]
    work: Callable[[object], float]  # bytes (GB/s) or flops (TFLOP/s) of one call of op
    kernel_regex: str
    cpu_ref: Optional[Callable[[tuple], object]] = None  # the reference's CPU program
    cpu_sample: Optional[Callable[[tuple], tuple]] = None  # bounded part of the problem
    cpu_sample_desc: str = ""
    shard: Optional[Callable[[tuple, int, int], Optional[tuple]]] = None
    shard_desc: str = ""
    unshard: Optional[Callable[[list, int], list]] = None  # gathered flats -> full layout
    bound: str = "hbm"
    # Roofline of the dominant kernel when it is not in the metric's unit
    # (GDN: metric TFLOP/s, bound HBM): work per call in that unit.
    roof_unit: Optional[str] = None
    roof_work: Optional[Callable[[object], float]] = None
    launches_per_call: int = 1  # kernels of this library one call launches
    baseline: bool = True  # one of BASELINE.json's configs
    # ``work`` computed from input shapes alone, for ops whose eval_roofline
    # binds the shape in forward (the CPU legs never call our kernels).
    units: Optional[Callable[[tuple], float]] = None
    extra: dict = field(default_factory=dict)


def host_work(wl: Workload, inputs: tuple) -> float:
    """The op's algorithmic work for these inputs without launching it."""
    if wl.units is not None:
        return float(wl.units(inputs))
    return float(wl.work(wl.build_op(inputs)))


def _gen(dev, seed):
    return torch.Generator(device=dev).manual_seed(seed)


def _rows_shard(n_split: int):
    """Shard the first ``n_split`` inputs along axis 0, keep the rest whole."""

    def shard(inp, index, count):
        parts = [shard_axis0(t, index, count) for t in inp[:n_split]]
        if any(p is None for p in parts):
            return None
        return tuple(parts) + tuple(inp[n_split:])

    return shard


def _faln() -> Workload:
    from tileops.ops.norm import FusedAddLayerNormFwdOp

    M, N = 8192, 4096

    def make(dev, seed):
        g = _gen(dev, seed)
        x = torch.randn(M, N, generator=g, device=dev).to(torch.bfloat16)
        r = torch.randn(M, N, generator=g, device=dev).to(torch.bfloat16)
        w = 1.0 + 0.1 * torch.randn(N, generator=g, device=dev)
        b = 0.1 * torch.randn(N, generator=g, device=dev)
        return x, r, w, b

    def cpu(inp):
        from oracle import reference as ref

        return ref.fused_add_layer_norm(*inp)

    return Workload(
        name="fused_add_layer_norm", metric="achieved HBM GB/s (FusedAddLayerNormFwdOp)",
        unit="GB/s", dtype="bf16",
        config={"workload": "FusedAddLayerNormFwdOp x,residual (8192,4096) bf16 + fp32 "
                            "weight/bias (N=4096), eps 1e-5 (BASELINE configs[1])",
                "M": M, "N": N},
        make_inputs=make, build_op=lambda inp: FusedAddLayerNormFwdOp(dtype=torch.bfloat16),
        run=lambda op, inp: op(*inp), work=lambda op: float(op.eval_roofline()[1]),
        kernel_regex="faln_", cpu_ref=cpu, shard=_rows_shard(2), shard_desc="rows of M",
        units=lambda inp: (4 * inp[0].numel() * inp[0].element_size()
                           + 2 * inp[2].numel() * inp[2].element_size()),
    )


def _gated(tanh: bool) -> Workload:
    from tileops.ops.elementwise import GeluAndMulFwdOp, GeluTanhAndMulFwdOp

    M, N = 4096, 11008
    cls = GeluTanhAndMulFwdOp if tanh else GeluAndMulFwdOp

    def make(dev, seed):
        return (torch.randn(M, 2 * N, generator=_gen(dev, seed), device=dev).to(torch.bfloat16),)

    def cpu(inp):
        from oracle import reference as ref

        return (ref.gelu_tanh_and_mul if tanh else ref.gelu_and_mul)(inp[0])

    name = "gelu_tanh_and_mul" if tanh else "gelu_and_mul"
    return Workload(
        name=name, metric=f"achieved HBM GB/s ({cls.__name__})", unit="GB/s", dtype="bf16",
        config={"workload": f"{cls.__name__} x (4096, 22016) bf16 -> (4096, 11008) "
                            "(BASELINE configs[0])", "M": M, "N": N},
        make_inputs=make, build_op=lambda inp: cls(inp[0].shape[0], N, torch.bfloat16),
        run=lambda op, inp: op(*inp), work=lambda op: float(op.eval_roofline()[1]),
        kernel_regex="gated_vec", cpu_ref=cpu, shard=_rows_shard(1), shard_desc="rows of M",
    )


def _unary(kind: str) -> Workload:
    from tileops.ops import elementwise as E

    shape = (16384, 16384)
    dtype = torch.int32 if kind == "bitwise_not" else torch.bfloat16
    op_cls = {"hardswish": E.HardswishFwdOp, "hardsigmoid": E.HardsigmoidFwdOp,
              "clamp_scalar": E.ClampScalarFwdOp, "isnan": E.IsnanFwdOp,
              "isinf": E.IsinfFwdOp, "isfinite": E.IsfiniteFwdOp,
              "bitwise_not": E.BitwiseNotFwdOp}[kind]

    def build(inp):
        n = inp[0].numel()
        if kind == "clamp_scalar":
            return op_cls(n, dtype, min=-0.5, max=0.5)
        return op_cls(n, dtype)

    def make(dev, seed):
        g = _gen(dev, seed)
        if dtype == torch.int32:
            return (torch.randint(-128, 128, shape, generator=g, device=dev, dtype=torch.int32),)
        x = torch.randn(shape, generator=g, device=dev).to(dtype)
        if kind.startswith("is"):
            # The reference's quarter draw (workloads/elementwise.py:103-111).
            q = x.numel() // 4
            f = x.view(-1)
            f[:q], f[q : 2 * q], f[2 * q : 3 * q] = float("nan"), float("inf"), float("-inf")
        return (x,)

    def cpu(inp):
        # The reference tests' own torch programs (test_<op>.py ref_program).
        import torch.nn.functional as F

        x = inp[0]
        if kind == "hardswish":
            return F.hardswish(x.float()).to(dtype)
        if kind == "hardsigmoid":
            return F.hardsigmoid(x.float()).to(dtype)
        if kind == "clamp_scalar":
            return torch.clamp(x.float(), -0.5, 0.5).to(dtype)
        if kind == "bitwise_not":
            return torch.bitwise_not(x)
        return getattr(torch, kind)(x.float())

    return Workload(
        name=kind, metric=f"achieved HBM GB/s ({op_cls.__name__})", unit="GB/s",
        dtype=str(dtype).split(".")[-1],
        config={"workload": f"{op_cls.__name__} [16384, 16384] {str(dtype).split('.')[-1]}"
                + (" (a quarter each NaN, +Inf, -Inf, randn)" if kind.startswith("is") else "")},
        make_inputs=make, build_op=build, run=lambda op, inp: op(*inp),
        work=lambda op: float(op.eval_roofline()[1]),
        kernel_regex="predicate_vec" if kind.startswith("is") else
        ("xor_stream_vec" if kind == "bitwise_not" else "unary_map_vec"),
        cpu_ref=cpu, shard=_rows_shard(1), shard_desc="rows of the [16384, 16384] input",
    )


def _causal_conv(activation) -> Workload:
    from tileops.ops.convolution import CausalDepthwiseConv1dFwdOp

    B, D, L, K = 8, 4096, 8192, 4

    def make(dev, seed):
        g = _gen(dev, seed)
        x = torch.randn(B, D, L, generator=g, device=dev).to(torch.bfloat16)
        w = (0.5 * torch.randn(D, K, generator=g, device=dev)).to(torch.bfloat16)
        b = (0.1 * torch.randn(D, generator=g, device=dev)).to(torch.bfloat16)
        return x, w, b

    def cpu(inp):
        from oracle import reference as ref

        return ref.causal_depthwise_conv1d(*inp, activation=activation)

    return Workload(
        name="causal_conv1d" + ("_silu" if activation else ""),
        metric="achieved HBM GB/s (CausalDepthwiseConv1dFwdOp)", unit="GB/s", dtype="bf16",
        config={"workload": f"causal depthwise conv1d x (8, 4096, 8192) bf16, w (4096, 4), "
                            f"bias, left pad 3, activation={activation} (BASELINE configs[2])"},
        make_inputs=make,
        build_op=lambda inp: CausalDepthwiseConv1dFwdOp(activation=activation),
        run=lambda op, inp: op(*inp), work=lambda op: float(op.eval_roofline()[1]),
        kernel_regex="dwconv_packet", cpu_ref=cpu, shard=_rows_shard(1), shard_desc="batch",
        units=lambda inp: (2 * inp[0].numel() * inp[0].element_size()
                           + inp[1].numel() * inp[1].element_size()
                           + inp[2].numel() * inp[2].element_size()),
    )


def _mha(causal: bool) -> Workload:
    from tileops.ops.attention import MultiHeadAttentionFwdOp

    B, S, H, D = 8, 4096, 32, 128

    def make(dev, seed):
        g = _gen(dev, seed)
        return tuple(torch.randn(B, S, H, D, generator=g, device=dev).to(torch.bfloat16)
                     for _ in range(3))

    def cpu(inp):
        from oracle import reference as ref

        return ref.mha_sdpa(*inp, causal)

    return Workload(
        name="mha_causal" if causal else "mha", unit="TFLOP/s", dtype="bf16", bound="tensor",
        metric="achieved TFLOP/s (MultiHeadAttentionFwdOp)",
        config={"workload": f"MultiHeadAttentionFwdOp q/k/v (8, 4096, 32, 128) bf16 BSHD, "
                            f"causal={causal}, scale 1/sqrt(128) (BASELINE configs[3])"},
        make_inputs=make,
        build_op=lambda inp: MultiHeadAttentionFwdOp(inp[0].shape[0], H, S, D, causal,
                                                     torch.bfloat16),
        run=lambda op, inp: op(*inp), work=lambda op: float(op.eval_roofline()[0]),
        kernel_regex="attn_fwd_kernel", cpu_ref=cpu, shard=_rows_shard(3),
        shard_desc="batch ((batch, head) pairs)",
    )


def _gdn() -> Workload:
    import torch.nn.functional as F

    from tileops.ops.linear_attention import GatedDeltaNetPrefillFwdOp

    B, T, H, DK, DV = 4, 8192, 16, 128, 128

    def make(dev, seed):
        g_ = _gen(dev, seed)
        q = F.normalize(torch.randn(B, T, H, DK, generator=g_, device=dev), dim=-1)
        k = F.normalize(torch.randn(B, T, H, DK, generator=g_, device=dev), dim=-1)
        v = torch.randn(B, T, H, DV, generator=g_, device=dev)
        g = F.logsigmoid(torch.randn(B, T, H, generator=g_, device=dev)) / 16
        beta = torch.sigmoid(torch.randn(B, T, H, generator=g_, device=dev))
        return (q.to(torch.bfloat16), k.to(torch.bfloat16), v.to(torch.bfloat16), g, beta)

    def shard(inp, index, count):  # of these inputs (the whole problem or a rank's part)
        sl = bh_split(inp[0].shape[0], inp[0].shape[2], index, count)
        if sl is None:
            return None
        bs, hs = sl
        return tuple(t[bs, :, hs].contiguous() for t in inp)

    def unshard(flats, count):
        return [unshard_bthd(flats[0], B, T, H, DV, count), flats[1].view(B, H, DK, DV)]

    def cpu(inp):
        from oracle import reference as ref

        return ref.gdn_prefill_bthd(*inp)

    return Workload(
        name="gdn", unit="TFLOP/s", dtype="bf16", bound="hbm", roof_unit="GB/s",
        roof_work=lambda op: float(op.eval_roofline()[1]),
        metric="achieved TFLOP/s (GatedDeltaNetPrefillFwdOp)",
        config={"workload": "GatedDeltaNetPrefillFwdOp B=4 T=8192 H=16 dk=dv=128 chunk 64, "
                            "q/k L2-normalised, g=logsigmoid(N)/16, beta=sigmoid(N), h0=0 "
                            "(BASELINE configs[4])"},
        make_inputs=make,
        build_op=lambda inp: GatedDeltaNetPrefillFwdOp(inp[0].shape[0], T, inp[0].shape[2],
                                                       DK, DV),
        run=lambda op, inp: op(*inp), work=lambda op: float(op.eval_roofline()[0]),
        kernel_regex="gdn_", cpu_ref=cpu, shard=shard, unshard=unshard,
        shard_desc="(batch, head) pairs", launches_per_call=2,  # gdn_prepare + gdn_scan
    )


def _gla() -> Workload:
    from tileops.ops.linear_attention import GLADecodeOp

    B, H, DK, DV = 8, 32, 128, 128

    def make(dev, seed):
        g = _gen(dev, seed)
        q = torch.randn(B, H, DK, generator=g, device=dev) * 0.5
        k = torch.randn(B, H, DK, generator=g, device=dev) * 0.5
        v = torch.randn(B, H, DV, generator=g, device=dev) * 0.5
        gk = -torch.rand(B, H, DK, generator=g, device=dev)
        state = torch.randn(B, H, DK, DV, generator=g, device=dev)
        return tuple(t.to(torch.bfloat16) for t in (q, k, v, gk, state))

    def cpu(inp):
        from oracle import reference as ref

        return ref.gla_decode(*inp, DK ** -0.5)

    return Workload(
        name="gla_decode", metric="achieved HBM GB/s (GLADecodeOp)", unit="GB/s",
        dtype="bf16", baseline=False,
        config={"workload": "GLADecodeOp B=8 H=32 DK=DV=128 bf16, one decode step (the "
                            "reference test's largest serving case, serving-b8-h32)"},
        make_inputs=make,
        build_op=lambda inp: GLADecodeOp(inp[0].shape[0], H, DK, DV, dtype=torch.bfloat16),
        run=lambda op, inp: op(*inp), work=lambda op: float(op.eval_roofline()[1]),
        kernel_regex="gla_decode", cpu_ref=cpu, shard=_rows_shard(5), shard_desc="batch",
    )


def _ssd() -> Workload:
    from tileops.ops.mamba import SSDChunkScanFwdOp

    B, NC, Q, H, P, N, G = 4, 8, 256, 80, 64, 128, 1
    S = NC * Q

    def make(dev, seed):
        g = _gen(dev, seed)
        x = (torch.randn(B, S, H, P, generator=g, device=dev) * 0.1).to(torch.bfloat16)
        cb = (torch.randn(B, NC, G, Q, Q, generator=g, device=dev) * 0.1).to(torch.bfloat16)
        dA = -torch.rand(B, H, NC, Q, generator=g, device=dev).cumsum(-1)
        Cm = (torch.randn(B, S, G, N, generator=g, device=dev) * 0.1).to(torch.bfloat16)
        prev = torch.randn(B, NC, H, P, N, generator=g, device=dev) * 0.1
        dt = (torch.rand(B, H, NC, Q, generator=g, device=dev) * 0.1 + 0.01).to(torch.bfloat16)
        return x, cb, dA, Cm, prev, dt

    def cpu(inp):
        from oracle import reference as ref

        return ref.ssd_chunk_scan(*inp, G)

    def units(inp):  # the op's eval_roofline bytes from the input shapes
        x, cb, dA, Cm, prev, dt = inp
        b, s, h, p = x.shape
        tok, eb = b * s * h, x.element_size()
        return float(tok * p * eb + cb.numel() * eb + tok * 4 + Cm.numel() * eb
                     + prev.numel() * 4 + tok * eb + tok * p * 4)

    return Workload(
        name="ssd_chunk_scan", metric="achieved HBM GB/s (SSDChunkScanFwdOp)", unit="GB/s",
        dtype="bf16", baseline=False,
        config={"workload": "SSDChunkScanFwdOp x (4, 2048, 80, 64) bf16, chunk 256, d_state "
                            "128, 1 group (manifest mamba2-2p7b-b4-s2k)"},
        make_inputs=make, build_op=lambda inp: SSDChunkScanFwdOp(),
        run=lambda op, inp: op(*inp), work=lambda op: float(op.eval_roofline()[1]),
        kernel_regex="ssd_chunk_scan", cpu_ref=cpu, shard=_rows_shard(6), shard_desc="batch",
        units=units,
    )


def _conv_dense() -> Workload:
    from tileops.ops.convolution import Conv1dBiasFwdOp

    N, CI, L, CO, K = 1, 80, 3000, 1280, 3

    def make(dev, seed):
        g = _gen(dev, seed)
        x = torch.randn(N, CI, L, generator=g, device=dev).to(torch.float16)
        w = (torch.randn(CO, CI, K, generator=g, device=dev) * 0.1).to(torch.float16)
        b = (torch.randn(CO, generator=g, device=dev) * 0.1).to(torch.float16)
        return x, w, b

    def cpu(inp):
        from oracle import reference as ref

        return ref.conv1d(inp[0], inp[1], inp[2], 1, 0, 1, 1)

    return Workload(
        name="conv1d_dense", unit="TFLOP/s", dtype="f16", bound="tensor", baseline=False,
        metric="achieved TFLOP/s (Conv1dBiasFwdOp, dense)",
        config={"workload": "Conv1dBiasFwdOp x (1, 80, 3000) f16, weight (1280, 80, 3), bias, "
                            "stride 1, no padding (manifest whisper-conv1-bias)"},
        make_inputs=make, build_op=lambda inp: Conv1dBiasFwdOp(),
        run=lambda op, inp: op(*inp), work=lambda op: float(op.eval_roofline()[0]),
        kernel_regex="conv1d_igemm", cpu_ref=cpu, shard=None,
        # 2 flops per tap (valid padding: every one of the K taps of every
        # output is in range) + 1 per output for the bias.
        units=lambda inp: float(N * CO * (L - K + 1) * (2 * CI * K + 1)),
    )


def _gdn_varlen() -> Workload:
    import torch.nn.functional as F

    from tileops.ops.linear_attention import GatedDeltaNetPrefillFwdOp

    TOTAL, H, DK, DV = 4 * 8192, 16, 128, 128
    # 12 sequences of ragged lengths (seeded), 32768 tokens in all: the
    # BASELINE token count packed fla-style (batch 1, cu_seqlens).
    gl = torch.Generator(device="cpu").manual_seed(7)
    cuts = sorted(torch.randint(1, TOTAL, (11,), generator=gl).tolist())
    offsets = [0] + cuts + [TOTAL]

    def make(dev, seed):
        g_ = _gen(dev, seed)
        q = F.normalize(torch.randn(1, TOTAL, H, DK, generator=g_, device=dev), dim=-1)
        k = F.normalize(torch.randn(1, TOTAL, H, DK, generator=g_, device=dev), dim=-1)
        v = torch.randn(1, TOTAL, H, DV, generator=g_, device=dev)
        g = F.logsigmoid(torch.randn(1, TOTAL, H, generator=g_, device=dev)) / 16
        beta = torch.sigmoid(torch.randn(1, TOTAL, H, generator=g_, device=dev))
        cu = torch.tensor(offsets, dtype=torch.int32, device=dev)
        return (q.to(torch.bfloat16), k.to(torch.bfloat16), v.to(torch.bfloat16), g, beta, cu)

    def cpu(inp):
        from oracle import reference as ref

        return ref.gdn_prefill_varlen(*inp[:5], inp[5])

    def sample(inp):  # the first sequence, all heads
        t = offsets[1]
        return tuple(x[:, :t].contiguous() for x in inp[:5]) + (
            torch.tensor([0, t], dtype=torch.int32),)

    return Workload(
        name="gdn_varlen", unit="TFLOP/s", dtype="bf16", bound="hbm", roof_unit="GB/s",
        roof_work=lambda op: float(op.eval_roofline()[1]), baseline=False,
        metric="achieved TFLOP/s (GatedDeltaNetPrefillFwdOp, packed cu_seqlens)",
        config={"workload": "GatedDeltaNetPrefillFwdOp packed: 32768 tokens (the BASELINE "
                            "token count) in 12 seeded ragged sequences, H=16 dk=dv=128, "
                            "chunk 64, same input distributions as the BASELINE config",
                "cu_seqlens": offsets},
        make_inputs=make,
        build_op=lambda inp: GatedDeltaNetPrefillFwdOp(1, inp[0].shape[1], H, DK, DV),
        run=lambda op, inp: op(*inp[:5], None, cu_seqlens=inp[5]),
        work=lambda op: float(op.eval_roofline()[0]),
        kernel_regex="gdn_", cpu_ref=cpu, cpu_sample=sample,
        cpu_sample_desc=f"the first packed sequence ({offsets[1]} tokens, all 16 heads)",
        shard=None, launches_per_call=3,  # chunk index + prepare + scan
    )


def workloads() -> dict[str, Callable[[], Workload]]:
    table = {
        "fused_add_layer_norm": _faln,
        "gelu_and_mul": lambda: _gated(False),
        "gelu_tanh_and_mul": lambda: _gated(True),
    }
    for kind in ("hardswish", "hardsigmoid", "clamp_scalar", "isnan", "isinf", "isfinite",
                 "bitwise_not"):
        table[kind] = (lambda k: (lambda: _unary(k)))(kind)
    table.update({
        "causal_conv1d": lambda: _causal_conv(None),
        "causal_conv1d_silu": lambda: _causal_conv("silu"),
        "mha": lambda: _mha(False),
        "mha_causal": lambda: _mha(True),
        "gdn": _gdn,
        "gdn_varlen": _gdn_varlen,
        "gla_decode": _gla,
        "ssd_chunk_scan": _ssd,
        "conv1d_dense": _conv_dense,
    })
    return table


# --------------------------------------------------------------- utilities
def load_peaks() -> tuple[dict, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        try:
            return json.loads(path.read_text()), "measured"
        except ValueError:
            pass
    return dict(FALLBACK_PEAKS), "fallback"


def load_traffic(name: str) -> Optional[float]:
    """DRAM bytes per launch of the op's dominant kernel from the committed
    ncu summary (a static capture, not a measurement of this run)."""
    path = ROOT / "profiles" / "ncu_traffic.json"
    if not path.exists():
        return None
    try:
        entry = json.loads(path.read_text()).get(name)
    except ValueError:
        return None
    return None if entry is None else float(entry["bytes_per_launch"])


class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML on a thread."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
        0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
    }

    def __init__(self, device_index: int, period_s: float = 0.005):
        self.samples: list[tuple[int, int]] = []
        self.max_mhz: Optional[int] = None
        self.period = period_s
        self._stop = threading.Event()
        self._thread = None
        self._handle = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nvml = pynvml
            uuid = None
            try:
                uuid = torch.cuda.get_device_properties(device_index).uuid
            except Exception:
                pass
            handle = None
            if uuid is not None:
                for i in range(pynvml.nvmlDeviceGetCount()):
                    h = pynvml.nvmlDeviceGetHandleByIndex(i)
                    if str(uuid) in str(pynvml.nvmlDeviceGetUUID(h)):
                        handle = h
            self._handle = handle or pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._handle, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._nvml = None

    def _sample(self):
        n = self._nvml
        sm = n.nvmlDeviceGetClockInfo(self._handle, n.NVML_CLOCK_SM)
        reasons = n.nvmlDeviceGetCurrentClocksEventReasons(self._handle)
        self.samples.append((sm, reasons))

    def _loop(self):
        while not self._stop.is_set():
            try:
                self._sample()
            except Exception:
                return
            time.sleep(self.period)

    def __enter__(self):
        if self._nvml is not None:
            self._stop.clear()
            self._thread = threading.Thread(target=self._loop, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join()
            self._thread = None
            try:
                self._sample()
            except Exception:
                pass

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unsampled"]}
        busy = [s for s in self.samples if not (s[1] & 0x1)] or self.samples
        reasons = set()
        for _, r in busy:
            for bit, name in self.REASONS.items():
                if r & bit and bit != 0x1:
                    reasons.add(name)
        return {"sm_mhz": statistics.median(s[0] for s in busy), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(reasons), "samples": len(busy)}


def dist_env() -> tuple[int, int, int]:
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)),
            int(os.environ.get("WORLD_SIZE", 1)))


def max_over_ranks(value: float, world: int, device) -> float:
    if world == 1:
        return value
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int, device) -> None:
    if world > 1:
        import torch.distributed as dist

        if device.type == "cuda":
            dist.barrier(device_ids=[device.index])
        else:  # gloo ranks (host-side tests of the multi-rank path)
            dist.barrier()


def check_shard_shapes(shapes: list[tuple], world: int, device) -> None:
    """Every rank must hold shards of the same shapes before an all-gather
    (``all_gather_into_tensor`` needs equal sizes): exchange the shapes and
    raise on every rank, naming the ranks, if they differ."""
    if world == 1:
        return
    import torch.distributed as dist

    flat = [len(shapes)] + [len(s) for s in shapes] + [d for s in shapes for d in s]
    width = torch.tensor([len(flat)], dtype=torch.int64, device=device)
    widths = [torch.zeros_like(width) for _ in range(world)]
    dist.all_gather(widths, width)
    n = int(max(w.item() for w in widths))
    mine = torch.full((n,), -1, dtype=torch.int64, device=device)
    mine[: len(flat)] = torch.tensor(flat, dtype=torch.int64, device=device)
    every = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(every, mine)
    ref = every[0]
    bad = [r for r in range(world) if not torch.equal(every[r], ref)]
    if bad:
        raise RuntimeError(f"shard shapes differ between rank 0 and ranks {bad}: "
                           f"{[e.tolist() for e in every]}")


def gather_outputs(outs, world: int, device, fulls=None):
    """Reassemble every rank's output shards on every rank: one
    ``all_gather_into_tensor`` per output (NCCL over NVLink on GPUs, gloo
    on CPU ranks), into ``fulls`` (allocated when None).  Shards land in
    rank order.  Returns the gathered flat tensors."""
    import torch.distributed as dist

    flats = [o.contiguous().view(-1) for o in outs]
    if fulls is None:
        fulls = [torch.empty(world * f.numel(), dtype=f.dtype, device=f.device) for f in flats]
    for full, flat in zip(fulls, flats):
        dist.all_gather_into_tensor(full, flat)
    return fulls


def whole_job_value(work_per_step: float, steps: int, total_ms: float, unit: str) -> float:
    """Throughput of ``steps`` steps of ``work_per_step`` units (summed over
    ranks) in ``total_ms`` (the slowest rank's timed region)."""
    scale = 1e9 if unit == "GB/s" else 1e12
    return work_per_step * steps / (total_ms * 1e-3) / scale


def _nbytes(ts) -> int:
    return sum(t.numel() * t.element_size() for t in ts if isinstance(t, torch.Tensor))


def _as_tuple(out) -> tuple:
    return tuple(out) if isinstance(out, (tuple, list)) else (out,)


def _problem(wl: Workload, device, seed: int, rank: int, world: int, pieces: int = 1) -> list:
    """The rank's part of the problem drawn from ``seed`` as a list of input
    tuples: ``[whole problem]`` at N = 1; else the problem is cut into
    ``world * pieces`` equal parts and rank r owns parts r, world + r, ...
    (so the i-th part of every rank, gathered in rank order, is a contiguous
    run of the whole problem)."""
    full = wl.make_inputs(device, seed)
    if world == 1:
        return [full]
    count = world * pieces
    mine = [wl.shard(full, i * world + rank, count) if wl.shard else None
            for i in range(pieces)]
    if any(m is None for m in mine):
        raise RuntimeError(f"{wl.name}: the problem does not split into {count} equal parts")
    del full
    return mine


# -------------------------------------------------------------- timing legs
def time_calls(run: Callable, sets: list, steps: int, warmup: int, graph: bool,
               device, stream) -> dict:
    """K steps over rotating input sets, a step being ``run(set)`` (the op on
    every part of the rank's problem): graph replays (or eager steps) with
    CUDA events around each; returns total and mean per-step ms."""
    n_sets = len(sets)
    for i in range(warmup):
        run(sets[i % n_sets])
    torch.cuda.synchronize(device)
    out_bytes = max(1, _nbytes(run(sets[0])))
    per_graph = max(1, min(64, (8 << 30) // out_bytes) // n_sets) * n_sets
    per_graph = min(per_graph, steps)

    def capture(n):
        g = torch.cuda.CUDAGraph()
        keep = []
        with torch.cuda.graph(g):
            for i in range(n):
                keep.append(run(sets[i % n_sets]))
        del keep
        return g

    graphs = []
    if graph:
        g_main = capture(per_graph)
        graphs.append(g_main)
        rem = steps % per_graph
        chunks = [(g_main.replay, per_graph)] * (steps // per_graph)
        if rem:
            g_rem = capture(rem)
            graphs.append(g_rem)
            chunks.append((g_rem.replay, rem))
        for _ in range(max(1, -(-warmup // per_graph))):
            g_main.replay()
        torch.cuda.synchronize(device)
    else:
        chunks = [((lambda inp=sets[i % n_sets]: run(inp)), 1) for i in range(steps)]
    starts = [torch.cuda.Event(enable_timing=True) for _ in chunks]
    ends = [torch.cuda.Event(enable_timing=True) for _ in chunks]
    torch.cuda.synchronize(device)
    for i, (fn, _) in enumerate(chunks):
        starts[i].record(stream)
        fn()
        ends[i].record(stream)
    torch.cuda.synchronize(device)
    total = starts[0].elapsed_time(ends[-1])
    per_call = sum(s.elapsed_time(e) for s, e in zip(starts, ends)) / steps
    calls = chunks[0][1]
    del chunks, graphs
    return {"total_ms": total, "per_call_ms": per_call, "calls_per_replay": calls}


def time_sharded_steps(wl: Workload, op, sets: list, steps: int, warmup: int, world: int,
                       device, stream) -> dict:
    """K steps of (the op on each part this rank owns, every part's outputs
    gathered on every rank as soon as that part is done, then the full layout
    back), eager, CUDA events around all K steps on the launching stream.
    With several parts the gather of part i (NCCL, asynchronous) runs while
    the op computes part i + 1."""
    import torch.distributed as dist

    n_sets, parts = len(sets), len(sets[0])
    outs = [_as_tuple(wl.run(op, part)) for part in sets[0]]
    check_shard_shapes([tuple(o.shape) for o in outs[0]], world, device)
    numels = [o.numel() for o in outs[0]]
    fulls = [torch.empty(world * parts * n, dtype=o.dtype, device=device)
             for o, n in zip(outs[0], numels)]

    def gather_part(i, res):
        works = []
        for full, o, n in zip(fulls, res, numels):
            dst = full[i * world * n:(i + 1) * world * n]
            works.append(dist.all_gather_into_tensor(dst, o.contiguous().view(-1),
                                                     async_op=True))
        return works

    def finish(works):
        for w in works:
            w.wait()
        if wl.unshard is not None:
            wl.unshard(fulls, world * parts)

    def step(i):
        works = []
        for j, part in enumerate(sets[i % n_sets]):
            works += gather_part(j, _as_tuple(wl.run(op, part)))
        finish(works)

    for i in range(max(1, warmup)):
        step(i)
    torch.cuda.synchronize(device)
    barrier(world, device)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(steps):
        step(i)
    e1.record(stream)
    torch.cuda.synchronize(device)
    step_ms = e0.elapsed_time(e1) / steps
    # The reassembly alone, for the breakdown.
    barrier(world, device)
    g0 = torch.cuda.Event(enable_timing=True)
    g1 = torch.cuda.Event(enable_timing=True)
    reps = max(3, min(steps, 10))
    g0.record(stream)
    for _ in range(reps):
        works = []
        for j in range(parts):
            works += gather_part(j, outs[j])
        finish(works)
    g1.record(stream)
    torch.cuda.synchronize(device)
    gather_ms = g0.elapsed_time(g1) / reps
    per_rank = sum(_nbytes(o) for o in outs)
    return {"step_ms": step_ms, "gather_ms": gather_ms, "bytes_per_rank": per_rank,
            "bytes_total": world * per_rank, "bytes_received_per_rank": (world - 1) * per_rank,
            "parts_per_rank": parts}


def time_e2e(wl: Workload, host_full: tuple, device, steps: int, max_chunks: int = 4,
             copy_streams: int = 1) -> dict:
    """The public op API from pinned host buffers, chunked so that copies in
    both directions overlap the kernels: per chunk, H2D on an input stream,
    the op on the compute stream, D2H of its outputs on an output stream
    (``copy_streams`` streams each way, chunks dealt round-robin).  Returns ms
    per step (all chunks) and the bytes copied each way."""
    # A chunk costs ~0.1 ms of host time (op call, copies, events): no chunk
    # gets less than 4 MB of input.
    in_bytes = sum(t.numel() * t.element_size() for t in host_full if isinstance(t, torch.Tensor))
    max_chunks = max(1, min(max_chunks, in_bytes // (4 << 20)))
    n_chunks = 1
    for c in (max_chunks, 16, 8, 4, 2):
        if c <= max_chunks and wl.shard is not None and wl.shard(host_full, 0, c) is not None:
            n_chunks = c
            break
    if n_chunks == 1:
        parts = [host_full]
    else:
        parts = [wl.shard(host_full, i, n_chunks) for i in range(n_chunks)]
    host_in = [tuple(t.pin_memory() if isinstance(t, torch.Tensor) else t for t in p)
               for p in parts]
    dev_in = [tuple(torch.empty(t.shape, dtype=t.dtype, device=device)
                    if isinstance(t, torch.Tensor) else t for t in p) for p in host_in]
    op = wl.build_op(dev_in[0])
    for d, h in zip(dev_in, host_in):
        for dt, ht in zip(d, h):
            if isinstance(dt, torch.Tensor):
                dt.copy_(ht)
    first = _as_tuple(wl.run(op, dev_in[0]))
    host_out = [tuple(torch.empty(o.shape, dtype=o.dtype, pin_memory=True) for o in first)
                for _ in range(n_chunks)]
    del first
    s_ins = [torch.cuda.Stream(device) for _ in range(copy_streams)]
    s_comp = torch.cuda.Stream(device)
    s_outs = [torch.cuda.Stream(device) for _ in range(copy_streams)]
    ev_in = [torch.cuda.Event() for _ in range(n_chunks)]
    ev_done = [torch.cuda.Event() for _ in range(n_chunks)]
    torch.cuda.synchronize(device)

    def one_step():
        for i in range(n_chunks):
            s_in, s_out = s_ins[i % copy_streams], s_outs[i % copy_streams]
            with torch.cuda.stream(s_in):
                s_in.wait_event(ev_done[i])  # the previous step's call read these buffers
                for dt, ht in zip(dev_in[i], host_in[i]):
                    if isinstance(dt, torch.Tensor):
                        dt.copy_(ht, non_blocking=True)
                ev_in[i].record(s_in)
            with torch.cuda.stream(s_comp):
                s_comp.wait_event(ev_in[i])
                res = _as_tuple(wl.run(op, dev_in[i]))
                ev_done[i].record(s_comp)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev_done[i])
                for h, d in zip(host_out[i], res):
                    d.record_stream(s_out)
                    h.copy_(d, non_blocking=True)
            del res

    for _ in range(2):
        one_step()
    torch.cuda.synchronize(device)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    # One copy stream each way: the end of every step (its last D2H) is
    # stamped on the output stream, and the step time is the median interval
    # between consecutive stamps (steady state; a host hiccup of one step
    # does not move it).  Several copy streams: the mean over all steps.
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    e0.record(s_comp)
    for st in s_ins + s_outs:
        st.wait_stream(s_comp)
    for i in range(steps):
        one_step()
        if copy_streams == 1:
            ends[i].record(s_outs[0])
    for st in s_ins + s_outs:
        s_comp.wait_stream(st)
    e1.record(s_comp)
    torch.cuda.synchronize(device)
    ms = e0.elapsed_time(e1) / steps
    if copy_streams == 1 and steps >= 3:
        ms = statistics.median(a.elapsed_time(b) for a, b in zip(ends[:-1], ends[1:]))
    h2d = sum(_nbytes(h) for h in host_in)
    d2h = sum(_nbytes(h) for h in host_out)
    return {"ms_per_step": ms, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "chunks": n_chunks, "calls_per_step": n_chunks,
            "api": f"{type(op).__name__}.__call__ per chunk, pinned host buffers, "
                   f"H2D / op / D2H on {copy_streams} / 1 / {copy_streams} streams"}


def time_cpu(fn: Callable, inputs: tuple, budget_s: float = 10.0) -> tuple[float, int, bool]:
    """Seconds per call of ``fn(inputs)``: one call, then (when it took less
    than half the budget) up to 3 more within the budget, reporting their
    median.  Returns (seconds, timed calls, first call only)."""
    t0 = time.perf_counter()
    fn(inputs)
    first = time.perf_counter() - t0
    if first * 2 > budget_s:
        return first, 1, True
    times = []
    t_end = time.perf_counter() + budget_s
    while len(times) < 3 and (time.perf_counter() < t_end or len(times) < 1):
        t0 = time.perf_counter()
        fn(inputs)
        times.append(time.perf_counter() - t0)
    return statistics.median(times), len(times), False


def cpu_baseline(wl: Workload, full_cpu: tuple, work: float, budget_s: float = 10.0) -> dict:
    """The reference's torch CPU program on all host threads: the full
    configuration, or the workload's stated sample when it has one."""
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    if wl.cpu_sample is not None:
        inputs = wl.cpu_sample(full_cpu)
        units = host_work(wl, inputs)
        desc = f"sample: {wl.cpu_sample_desc}"
        same = False
    else:
        inputs, units, desc, same = full_cpu, work, "the full configuration", True
    sec, reps, cold = time_cpu(lambda inp: wl.cpu_ref(inp), inputs, budget_s)
    scale = 1e9 if wl.unit == "GB/s" else 1e12
    return {"value": units / sec / scale, "unit": wl.unit, "cores": torch.get_num_threads(),
            "kind": "port", "same_config": same, "ms_per_call": sec * 1e3,
            "sample": f"reference torch CPU program (restated in oracle/) on {desc}; "
                      + ("one cold call" if cold else f"median of {reps} calls after one"),
            "cpu_count": os.cpu_count()}


# ------------------------------------------------------------------ our arm
def _peak(unit: str, peaks: dict) -> tuple[float, str]:
    if unit == "GB/s":
        return float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"])), "GB/s"
    return float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"])), "TFLOP/s"


def measure(wl: Workload, args, rank: int, local_rank: int, world: int, device,
            with_cpu: bool, headline: bool) -> dict:
    """Every leg of one op: kernel-only replays, the sharded step with its
    reassembly (N > 1), the end-to-end host path, and the CPU baseline."""
    stream = torch.cuda.current_stream(device)
    pieces = args.pieces if world > 1 else 1
    try:
        probe = _problem(wl, device, SEED, rank, world, pieces)
    except RuntimeError:
        pieces = 1
        probe = _problem(wl, device, SEED, rank, world, pieces)
    op = wl.build_op(probe[0])

    def run(parts):  # the op on every part of this rank's problem
        return tuple(o for part in parts for o in _as_tuple(wl.run(op, part)))

    set_bytes = sum(_nbytes(p) for p in probe) + _nbytes(run(probe))
    n_sets = max(2, min(32, -(-3 * L2_BYTES // max(set_bytes, 1)) + 1))
    sets = [probe] + [_problem(wl, device, SEED + 1000 * i, rank, world, pieces)
                      for i in range(1, n_sets)]
    work = wl.work(op) * pieces  # this rank's part (all its pieces)
    peaks, peak_kind = load_peaks()
    roof_unit = wl.roof_unit or wl.unit
    roof_work = wl.roof_work(op) * pieces if wl.roof_work else work
    peak, peak_unit = _peak(roof_unit, peaks)
    steps = args.steps if headline else min(args.steps, args.per_op_steps)

    sampler = ClockSampler(local_rank)
    barrier(world, device)
    with sampler:
        k = time_calls(run, sets, steps, args.warmup, args.graph, device, stream)
        sharded = None
        if world > 1:
            sharded = time_sharded_steps(wl, op, sets, steps, args.warmup, world, device,
                                         stream)
    barrier(world, device)
    per_call_ms = max_over_ranks(k["per_call_ms"], world, device)
    total_ms = max_over_ranks(k["total_ms"], world, device)
    achieved = roof_work / (per_call_ms * 1e-3) / (1e9 if roof_unit == "GB/s" else 1e12)
    rec = {
        "metric": wl.metric, "unit": wl.unit, "dtype": wl.dtype, "config": dict(wl.config),
        "roofline": {"bound": wl.bound, "achieved": achieved, "peak": peak, "unit": peak_unit,
                     "frac": achieved / peak, "traffic": load_traffic(wl.name),
                     "traffic_source": "profiles/ncu_traffic.json (static ncu capture of "
                                       "this workload, not this run)",
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json)"
                     if peak_kind == "measured" else "fallback",
                     "per_launch_ms": per_call_ms, "algorithmic_per_launch": roof_work},
        "l2": f"rotating {n_sets} input/output sets ({n_sets * set_bytes / 2**20:.0f} MiB) "
              "> 126 MB L2",
        "timing": (f"CUDA-graph replays of {k['calls_per_replay']} op calls each, CUDA events "
                   "around each replay" if args.graph else "eager op calls"),
    }
    if world == 1:
        rec["value"] = whole_job_value(work, steps, total_ms, wl.unit)
        rec["ms_per_step"] = total_ms / steps
        rec["gpu_launches"] = steps * wl.launches_per_call
    else:
        step_ms = max_over_ranks(sharded["step_ms"], world, device)
        gather_ms = max_over_ranks(sharded["gather_ms"], world, device)
        rec["value"] = whole_job_value(world * work, 1, step_ms, wl.unit)
        rec["ms_per_step"] = step_ms
        rec["gpu_launches"] = steps * wl.launches_per_call
        rec["kernel_only"] = {
            "value": whole_job_value(world * work, 1, per_call_ms, wl.unit),
            "ms_per_step": per_call_ms,
            "note": "the op on this rank's parts alone, graph replays, slowest rank"}
        rec["gather"] = {
            "collective": "all_gather_into_tensor per output and part (NCCL, asynchronous: "
                          "part i is gathered while part i + 1 computes), then the full layout",
            "parts_per_rank": sharded["parts_per_rank"],
            "ms": gather_ms, "bytes_per_rank": sharded["bytes_per_rank"],
            "bytes_total": sharded["bytes_total"],
            "bytes_received_per_rank": sharded["bytes_received_per_rank"],
            "busbw_GBps": sharded["bytes_received_per_rank"] / (gather_ms * 1e-3) / 1e9}
        rec["config"]["parallelism"] = (
            f"{wl.shard_desc} split into {world} x {pieces} parts (same seed, sliced; rank r "
            f"owns parts r, {world} + r, ...) + NCCL all_gather_into_tensor reassembly"
            + (" overlapping the next part's op" if pieces > 1 else ""))
    rec["clocks"] = sampler.summary()

    # End to end through the public API from pinned host buffers: every part
    # of this rank's problem in turn.
    host_parts = [tuple(t.cpu() if isinstance(t, torch.Tensor) else t for t in part)
                  for part in sets[0]]
    del sets
    torch.cuda.empty_cache()
    e2e_steps = max(3, min(steps, 10))
    e2e_ms, h2d, d2h = 0.0, 0, 0
    for hp in host_parts:
        e = time_e2e(wl, hp, device, e2e_steps, args.e2e_chunks, args.e2e_streams)
        e2e_ms += e["ms_per_step"]
        h2d += e["h2d_bytes_per_step"]
        d2h += e["d2h_bytes_per_step"]
    e2e_ms = max_over_ranks(e2e_ms, world, device)
    rec["e2e"] = {"value": whole_job_value(world * work, 1, e2e_ms, wl.unit), "unit": wl.unit,
                  "h2d_bytes_per_step": h2d * world, "d2h_bytes_per_step": d2h * world,
                  "ms_per_step": e2e_ms, "chunks_per_rank": e["chunks"] * len(host_parts),
                  "api": e["api"]}
    if with_cpu and world == 1 and wl.cpu_ref is not None and rank == 0:
        rec["cpu_baseline"] = cpu_baseline(wl, host_parts[0], work, args.cpu_budget)
    del host_parts, probe, op
    torch.cuda.empty_cache()
    return rec


def _per_op_names(args, world: int, table: dict) -> list[str]:
    if args.per_op == "none":
        return []
    if args.per_op == "all":
        names = list(table)
    else:
        names = [n.strip() for n in args.per_op.split(",") if n.strip()]
        unknown = [n for n in names if n not in table]
        if unknown:
            raise SystemExit(f"unknown --per-op names {unknown}")
    if world > 1:  # the split BASELINE problems only
        names = [n for n in names if table[n]().baseline and table[n]().shard is not None]
    return [n for n in names if n != args.op]


def run_ours(args) -> Optional[dict]:
    rank, local_rank, world = dist_env()
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=args.pg_timeout),
                                device_id=device)
    table = workloads()
    wl = table[args.op]()
    head = measure(wl, args, rank, local_rank, world, device, not args.no_cpu_baseline, True)

    weak = None
    if world > 1 and not args.no_weak:
        # Secondary figure: every rank runs the whole problem (replicas).
        full = wl.make_inputs(device, SEED + rank)
        op = wl.build_op(full)
        n_sets = max(2, min(32, -(-3 * L2_BYTES // max(_nbytes(full) * 2, 1)) + 1))
        sets = [full] + [wl.make_inputs(device, SEED + rank + 1000 * i) for i in range(1, n_sets)]
        barrier(world, device)
        k = time_calls(lambda inp: _as_tuple(wl.run(op, inp)), sets,
                       min(args.steps, args.per_op_steps), args.warmup, args.graph, device,
                       torch.cuda.current_stream(device))
        barrier(world, device)
        ms = max_over_ranks(k["per_call_ms"], world, device)
        weak = {"value": whole_job_value(world * wl.work(op), 1, ms, wl.unit),
                "ms_per_step": ms, "note": "every rank runs the whole problem (replicas)"}
        del sets, full, op
        torch.cuda.empty_cache()

    per_op = {}
    for name in _per_op_names(args, world, table):
        per_op[name] = measure(table[name](), args, rank, local_rank, world, device,
                               not args.no_cpu_baseline, False)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    if rank != 0:
        return None
    line = {
        "metric": wl.metric, "value": head["value"], "unit": wl.unit, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": head["ms_per_step"],
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": wl.dtype,
        "data": "synthetic (seeded torch.randn of the BASELINE shapes)",
        "config": {**head["config"], "l2": head["l2"], "timing": head["timing"]},
        "roofline": head["roofline"], "e2e": head["e2e"],
        "gpu_launches": head["gpu_launches"], "clocks": head["clocks"],
    }
    line["config"].setdefault("parallelism", "dp1 (one GPU, the whole problem)")
    for key in ("kernel_only", "gather", "cpu_baseline"):
        if key in head:
            line[key] = head[key]
    if weak is not None:
        line["weak"] = weak
    line["per_op"] = {wl.name: _compact(head), **{n: _compact(r) for n, r in per_op.items()}}
    return line


def _compact(rec: dict) -> dict:
    out = {"value": rec["value"], "unit": rec["unit"], "ms_per_step": rec["ms_per_step"],
           "workload": rec["config"]["workload"],
           "roofline": {k: rec["roofline"][k] for k in ("bound", "achieved", "peak", "unit",
                                                         "frac", "traffic", "per_launch_ms")},
           "e2e": {k: rec["e2e"][k] for k in ("value", "ms_per_step", "h2d_bytes_per_step",
                                               "d2h_bytes_per_step", "chunks_per_rank")},
           "clocks": rec["clocks"], "gpu_launches": rec["gpu_launches"]}
    for key in ("kernel_only", "gather", "cpu_baseline"):
        if key in rec:
            out[key] = rec[key]
    return out


# ----------------------------------------------------------- reference arm
def run_reference(args) -> Optional[dict]:
    """The reference's CPU program (its tests' torch ref_program, restated in
    oracle/) on the host cores, rank 0 only: K timed calls after W warm-up
    calls on the headline op's full configuration, and at N = 1 every other
    op's CPU baseline under ``per_op``."""
    rank, _, world = dist_env()
    if rank != 0:
        return None
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    table = workloads()
    wl = table[args.op]()
    cpu = torch.device("cpu")
    full = wl.make_inputs(cpu, SEED)
    inputs = wl.cpu_sample(full) if wl.cpu_sample else full
    units = host_work(wl, inputs)
    for _ in range(args.warmup):
        wl.cpu_ref(inputs)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        wl.cpu_ref(inputs)
    sec = (time.perf_counter() - t0) / args.steps
    scale = 1e9 if wl.unit == "GB/s" else 1e12
    value = units / sec / scale
    desc = (f"sample: {wl.cpu_sample_desc}" if wl.cpu_sample else "the full configuration")
    line = {
        "impl": "reference", "metric": wl.metric, "value": value, "unit": wl.unit,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": sec * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": wl.dtype,
        "data": "synthetic (seeded torch.randn of the BASELINE shapes)",
        "config": {**wl.config, "parallelism": "host CPU, rank 0 only"},
        "cpu_baseline": {"value": value, "unit": wl.unit, "cores": torch.get_num_threads(),
                         "kind": "port", "same_config": wl.cpu_sample is None,
                         "sample": f"reference torch CPU program (restated in oracle/) on "
                                   f"{desc}, every step"},
        "e2e": {"value": value, "unit": wl.unit, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    del full, inputs
    if world == 1 and args.per_op not in (None, "none"):
        per_op = {}
        names = list(table) if args.per_op == "all" else [
            n.strip() for n in args.per_op.split(",") if n.strip()]
        for name in names:
            if name == args.op:
                continue
            w = table[name]()
            if w.cpu_ref is None:
                continue
            f = w.make_inputs(cpu, SEED)
            per_op[name] = cpu_baseline(w, f, host_work(w, f), args.cpu_budget)
            del f
        line["per_op"] = per_op
    return line


def main() -> None:
    ap = argparse.ArgumentParser(description="B200 TileOPs hot-path benchmark")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--op", default="fused_add_layer_norm", help="the headline op")
    ap.add_argument("--per-op", default=None,
                    help="'all', 'none' or a comma list of ops measured beside the headline "
                         "(N > 1: the BASELINE ops among them).  Default: 'all' for our arm, "
                         "'none' for the reference arm (our line carries every op's CPU "
                         "baseline already)")
    ap.add_argument("--per-op-steps", type=int, default=20,
                    help="timed calls per op in per_op (the headline uses --steps)")
    ap.add_argument("--e2e-chunks", type=int, default=4,
                    help="chunks per step in the end-to-end leg (at most; 4 measured "
                         "fastest: each chunk costs ~0.1 ms of host time for the op call "
                         "and its copies; no chunk gets less than 4 MB of input)")
    ap.add_argument("--pieces", type=int, default=1,
                    help="N > 1: parts per rank; each part's outputs are gathered while the "
                         "next part computes (1 = one shard per rank, gathered after it; "
                         "measured faster than 2 or 4 parts at N = 2)")
    ap.add_argument("--e2e-streams", type=int, default=1,
                    help="copy streams per direction in the end-to-end leg")
    ap.add_argument("--cpu-budget", type=float, default=10.0,
                    help="seconds of CPU time per op for the CPU baseline")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-weak", action="store_true",
                    help="N > 1: skip the per-rank replica (weak scaling) figure")
    ap.add_argument("--pg-timeout", type=int, default=300,
                    help="process-group timeout in seconds (a rank that left ends the "
                         "others' next collective with an error after this long)")
    ap.add_argument("--no-graph", dest="graph", action="store_false",
                    help="time eager op calls instead of CUDA-graph replays")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    if args.per_op is None:
        args.per_op = "all" if args.impl == "ours" else "none"
    table = workloads()
    if args.op not in table:
        raise SystemExit(f"unknown --op {args.op}; choose from {sorted(table)}")
    line = run_reference(args) if args.impl == "reference" else run_ours(args)
    if line is not None:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
