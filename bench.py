"""Benchmark of the hot path on B200: one JSON line per run.

Default workload: FusedAddLayerNormFwdOp on x, residual
(8192, 4096) bf16 ~ N(0, 1) with fp32 weight = 1 + 0.1 N(0,1), bias =
0.1 N(0,1), eps 1e-5.  A step is one forward over that batch.  ``--op``
selects another hot-path op at its BASELINE configuration (used for the
per-op tables; the default line is the contract's headline).

Metric: achieved HBM GB/s = algorithmic bytes of the op (its eval_roofline
bytes) / time, summed over ranks (weak scaling: every rank runs its own
batch, no collective on the data path).  MHA / GDN lines report TFLOP/s.

Timing: W warm-up steps, then K steps bracketed by a barrier and
``torch.cuda.synchronize()``, CUDA events on the launching stream around
every graph replay, max over ranks.  The K steps run as replays of a CUDA
graph holding up to 64 consecutive op calls, each with its own outputs
(``--no-graph``: K eager calls, which the host's Python cost can starve when
a kernel is ~50 us).  Inputs rotate over enough distinct buffer sets
that every step's working set was evicted from the 126 MB L2 (the set count
is in ``config``).  ``e2e`` repeats the measurement through the public op API
with pinned HOST buffers: H2D of the inputs, the op, D2H of the outputs.

``--impl reference`` times the reference's CPU path (the torch ref program,
restated in ``oracle/``) on the host cores, rank 0 only.

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


# ----------------------------------------------------------------- workloads
@dataclass
class Workload:
    """One op at one configuration."""

    name: str
    metric: str
    unit: str  # "GB/s" or "TFLOP/s"
    dtype: str
    config: dict
    make_inputs: Callable[[torch.device, int], tuple]  # (device, seed) -> device tensors
    build_op: Callable[[], object]
    run: Callable[[object, tuple], object]
    work_per_step: Callable[[object], float]  # bytes (GB/s) or flops (TFLOP/s) per step
    kernel_regex: str
    cpu_fn: Optional[Callable[[tuple], object]] = None  # oracle on CPU tensors
    cpu_slice: Optional[Callable[[tuple, int], tuple]] = None  # bounded sample of the inputs
    cpu_units: Optional[Callable[[tuple], float]] = None  # work units of a sample
    bound: str = "hbm"
    # Roofline of the dominant kernel when it is not in the metric's unit
    # (GDN: metric TFLOP/s, bound HBM): work per step in that unit.
    roof_unit: Optional[str] = None
    roof_work_per_step: Optional[Callable[[object], float]] = None
    launches_per_step: int = 1  # kernels of this library one step launches
    extra: dict = field(default_factory=dict)


def _faln() -> Workload:
    from tileops.ops.norm import FusedAddLayerNormFwdOp

    M, N = 8192, 4096

    def make(dev, seed):
        g = torch.Generator(device="cpu").manual_seed(seed)
        x = torch.randn(M, N, generator=g).to(torch.bfloat16)
        r = torch.randn(M, N, generator=g).to(torch.bfloat16)
        w = 1.0 + 0.1 * torch.randn(N, generator=g)
        b = 0.1 * torch.randn(N, generator=g)
        return tuple(t.to(dev) for t in (x, r, w, b))

    def units(inp):
        m, n = inp[0].shape
        return 4.0 * m * n * 2 + 2 * n * 4

    def cpu(inp):
        from oracle import reference as ref

        return ref.fused_add_layer_norm(*inp)

    return Workload(
        name="fused_add_layer_norm", metric="achieved HBM GB/s (FusedAddLayerNormFwdOp)",
        unit="GB/s", dtype="bf16",
        config={"workload": "FusedAddLayerNormFwdOp x,residual (8192,4096) bf16 + fp32 "
                            "weight/bias (N=4096), eps 1e-5 (BASELINE configs[1])",
                "M": M, "N": N},
        make_inputs=make, build_op=lambda: FusedAddLayerNormFwdOp(dtype=torch.bfloat16),
        run=lambda op, inp: op(*inp), work_per_step=lambda op: float(op.eval_roofline()[1]),
        kernel_regex="faln_", cpu_fn=cpu,
        cpu_slice=lambda inp, rows: (inp[0][:rows], inp[1][:rows], inp[2], inp[3]),
        cpu_units=units,
    )


def _gated(tanh: bool) -> Workload:
    from tileops.ops.elementwise import GeluAndMulFwdOp, GeluTanhAndMulFwdOp

    M, N = 4096, 11008
    cls = GeluTanhAndMulFwdOp if tanh else GeluAndMulFwdOp

    def make(dev, seed):
        g = torch.Generator(device="cpu").manual_seed(seed)
        return (torch.randn(M, 2 * N, generator=g).to(torch.bfloat16).to(dev),)

    def cpu(inp):
        from oracle import reference as ref

        return (ref.gelu_tanh_and_mul if tanh else ref.gelu_and_mul)(inp[0])

    name = "gelu_tanh_and_mul" if tanh else "gelu_and_mul"
    return Workload(
        name=name, metric=f"achieved HBM GB/s ({cls.__name__})", unit="GB/s", dtype="bf16",
        config={"workload": f"{cls.__name__} x (4096, 22016) bf16 -> (4096, 11008) "
                            "(BASELINE configs[0])", "M": M, "N": N},
        make_inputs=make, build_op=lambda: cls(M, N, torch.bfloat16),
        run=lambda op, inp: op(*inp), work_per_step=lambda op: float(op.eval_roofline()[1]),
        kernel_regex="gated_vec", cpu_fn=cpu,
        cpu_slice=lambda inp, rows: (inp[0][:rows],),
        cpu_units=lambda inp: 3.0 * inp[0].shape[0] * (inp[0].shape[1] // 2) * 2,
    )


def _unary(kind: str) -> Workload:
    from tileops.ops import elementwise as E

    shape = (16384, 16384)
    n = shape[0] * shape[1]
    dtype = torch.int32 if kind == "bitwise_not" else torch.bfloat16
    op_cls = {"hardswish": E.HardswishFwdOp, "hardsigmoid": E.HardsigmoidFwdOp,
              "clamp_scalar": E.ClampScalarFwdOp, "isnan": E.IsnanFwdOp,
              "isinf": E.IsinfFwdOp, "isfinite": E.IsfiniteFwdOp,
              "bitwise_not": E.BitwiseNotFwdOp}[kind]

    def build():
        if kind == "clamp_scalar":
            return op_cls(n, dtype, min=-0.5, max=0.5)
        return op_cls(n, dtype)

    def make(dev, seed):
        g = torch.Generator(device="cpu").manual_seed(seed)
        if dtype == torch.int32:
            x = torch.randint(-128, 128, shape, generator=g, dtype=torch.int32)
        else:
            x = torch.randn(shape, generator=g).to(dtype)
            if kind.startswith("is"):
                q = n // 4
                f = x.view(-1)
                f[:q], f[q : 2 * q], f[2 * q : 3 * q] = float("nan"), float("inf"), float("-inf")
        return (x.to(dev),)

    def cpu(inp):
        from oracle import reference as ref

        fn = getattr(ref, kind)
        return fn(inp[0], -0.5, 0.5) if kind == "clamp_scalar" else fn(inp[0])

    out_b = 1 if kind.startswith("is") else dtype.itemsize
    return Workload(
        name=kind, metric=f"achieved HBM GB/s ({op_cls.__name__})", unit="GB/s",
        dtype=str(dtype).split(".")[-1],
        config={"workload": f"{op_cls.__name__} [16384, 16384] {str(dtype).split('.')[-1]}"},
        make_inputs=make, build_op=build, run=lambda op, inp: op(*inp),
        work_per_step=lambda op: float(op.eval_roofline()[1]),
        kernel_regex="predicate_vec" if kind.startswith("is") else
        ("xor_stream_vec" if kind == "bitwise_not" else "unary_map_vec"),
        cpu_fn=cpu, cpu_slice=lambda inp, rows: (inp[0][:rows],),
        cpu_units=lambda inp: float(inp[0].numel() * (dtype.itemsize + out_b)),
    )


def _causal_conv(activation) -> Workload:
    from tileops.ops.convolution import CausalDepthwiseConv1dFwdOp

    B, D, L, K = 8, 4096, 8192, 4

    def make(dev, seed):
        g = torch.Generator(device="cpu").manual_seed(seed)
        x = torch.randn(B, D, L, generator=g).to(torch.bfloat16)
        w = (0.5 * torch.randn(D, K, generator=g)).to(torch.bfloat16)
        b = (0.1 * torch.randn(D, generator=g)).to(torch.bfloat16)
        return tuple(t.to(dev) for t in (x, w, b))

    def cpu(inp):
        from oracle import reference as ref

        return ref.causal_depthwise_conv1d(*inp, activation=activation)

    return Workload(
        name="causal_conv1d" + ("_silu" if activation else ""),
        metric="achieved HBM GB/s (CausalDepthwiseConv1dFwdOp)", unit="GB/s", dtype="bf16",
        config={"workload": f"causal depthwise conv1d x (8, 4096, 8192) bf16, w (4096, 4), "
                            f"bias, left pad 3, activation={activation} (BASELINE configs[2])"},
        make_inputs=make, build_op=lambda: CausalDepthwiseConv1dFwdOp(activation=activation),
        run=lambda op, inp: op(*inp), work_per_step=lambda op: float(op.eval_roofline()[1]),
        kernel_regex="dwconv_packet", cpu_fn=cpu,
        cpu_slice=lambda inp, rows: (inp[0][:1, : max(rows // 64, 1)],
                                     inp[1][: max(rows // 64, 1)], inp[2][: max(rows // 64, 1)]),
        cpu_units=lambda inp: 2.0 * inp[0].numel() * 2 + inp[1].numel() * 2 + inp[2].numel() * 2,
    )


def _mha(causal: bool) -> Workload:
    from tileops.ops.attention import MultiHeadAttentionFwdOp

    B, S, H, D = 8, 4096, 32, 128

    def make(dev, seed):
        g = torch.Generator(device="cpu").manual_seed(seed)
        return tuple(torch.randn(B, S, H, D, generator=g).to(torch.bfloat16).to(dev)
                     for _ in range(3))

    def cpu(inp):
        from oracle import reference as ref

        return ref.gqa_prefill_fwd(*inp, causal)

    def sample(inp, rows):
        s = max(128, min(S, rows * 4))
        return tuple(t[:1, :s, :1].contiguous() for t in inp)

    def units(inp):
        s = inp[0].shape[1]
        f = 4.0 * s * s * D
        return f / 2 if causal else f

    return Workload(
        name="mha_causal" if causal else "mha", unit="TFLOP/s", dtype="bf16", bound="tensor",
        metric="achieved TFLOP/s (MultiHeadAttentionFwdOp)",
        config={"workload": f"MultiHeadAttentionFwdOp q/k/v (8, 4096, 32, 128) bf16 BSHD, "
                            f"causal={causal}, scale 1/sqrt(128) (BASELINE configs[3])"},
        make_inputs=make,
        build_op=lambda: MultiHeadAttentionFwdOp(B, H, S, D, causal, torch.bfloat16),
        run=lambda op, inp: op(*inp), work_per_step=lambda op: float(op.eval_roofline()[0]),
        kernel_regex="attn_fwd_kernel", cpu_fn=cpu, cpu_slice=sample, cpu_units=units,
    )


def _gdn() -> Workload:
    import torch.nn.functional as F

    from tileops.ops.linear_attention import GatedDeltaNetPrefillFwdOp

    B, T, H, DK, DV = 4, 8192, 16, 128, 128

    def make(dev, seed):
        g_ = torch.Generator(device="cpu").manual_seed(seed)
        q = F.normalize(torch.randn(B, T, H, DK, generator=g_), dim=-1).to(torch.bfloat16)
        k = F.normalize(torch.randn(B, T, H, DK, generator=g_), dim=-1).to(torch.bfloat16)
        v = torch.randn(B, T, H, DV, generator=g_).to(torch.bfloat16)
        g = F.logsigmoid(torch.randn(B, T, H, generator=g_)) / 16
        beta = torch.sigmoid(torch.randn(B, T, H, generator=g_))
        return tuple(t.to(dev) for t in (q, k, v, g, beta))

    def cpu(inp):
        from oracle import reference as ref

        return ref.gdn_prefill_bthd(*inp)

    def sample(inp, rows):
        t = max(64, min(T, rows * 4))
        return tuple(x[:1, :t, :1].contiguous() for x in inp)

    def units(inp):
        t = inp[0].shape[1]
        return float(t * (4 * 64 * DK + 6 * DK * DV + 3 * 64 * DV))

    return Workload(
        name="gdn", unit="TFLOP/s", dtype="bf16", bound="hbm", roof_unit="GB/s",
        roof_work_per_step=lambda op: float(op.eval_roofline()[1]),
        metric="achieved TFLOP/s (GatedDeltaNetPrefillFwdOp)",
        config={"workload": "GatedDeltaNetPrefillFwdOp B=4 T=8192 H=16 dk=dv=128 chunk 64, "
                            "q/k L2-normalised, g=logsigmoid(N)/16, beta=sigmoid(N), h0=0 "
                            "(BASELINE configs[4])"},
        make_inputs=make,
        build_op=lambda: GatedDeltaNetPrefillFwdOp(B, T, H, DK, DV),
        run=lambda op, inp: op(*inp), work_per_step=lambda op: float(op.eval_roofline()[0]),
        kernel_regex="gdn_", cpu_fn=cpu, cpu_slice=sample, cpu_units=units,
        launches_per_step=2,  # gdn_prepare + gdn_scan
    )


def _gla() -> Workload:
    from tileops.ops.linear_attention import GLADecodeOp

    B, H, DK, DV = 8, 32, 128, 128

    def make(dev, seed):
        g = torch.Generator(device="cpu").manual_seed(seed)
        q = torch.randn(B, H, DK, generator=g) * 0.5
        k = torch.randn(B, H, DK, generator=g) * 0.5
        v = torch.randn(B, H, DV, generator=g) * 0.5
        gk = -torch.rand(B, H, DK, generator=g)
        state = torch.randn(B, H, DK, DV, generator=g)
        return tuple(t.to(torch.bfloat16).to(dev) for t in (q, k, v, gk, state))

    def cpu(inp):
        from oracle import reference as ref

        return ref.gla_decode(*inp, DK ** -0.5)

    def units(inp):
        b, h = inp[0].shape[:2]
        return float(b * h * (3 * DK + 2 * DV + 2 * DK * DV) * 2)

    return Workload(
        name="gla_decode", metric="achieved HBM GB/s (GLADecodeOp)", unit="GB/s",
        dtype="bf16",
        config={"workload": "GLADecodeOp B=8 H=32 DK=DV=128 bf16, one decode step (the "
                            "reference test's largest serving case, serving-b8-h32)"},
        make_inputs=make, build_op=lambda: GLADecodeOp(B, H, DK, DV, dtype=torch.bfloat16),
        run=lambda op, inp: op(*inp), work_per_step=lambda op: float(op.eval_roofline()[1]),
        kernel_regex="gla_decode", cpu_fn=cpu,
        cpu_slice=lambda inp, rows: tuple(t[:1] for t in inp), cpu_units=units,
    )


def _ssd() -> Workload:
    from tileops.ops.mamba import SSDChunkScanFwdOp

    B, NC, Q, H, P, N, G = 4, 8, 256, 80, 64, 128, 1
    S = NC * Q

    def make(dev, seed):
        g = torch.Generator(device="cpu").manual_seed(seed)
        x = (torch.randn(B, S, H, P, generator=g) * 0.1).to(torch.bfloat16)
        cb = (torch.randn(B, NC, G, Q, Q, generator=g) * 0.1).to(torch.bfloat16)
        dA = -torch.rand(B, H, NC, Q, generator=g).cumsum(-1)
        Cm = (torch.randn(B, S, G, N, generator=g) * 0.1).to(torch.bfloat16)
        prev = torch.randn(B, NC, H, P, N, generator=g) * 0.1
        dt = (torch.rand(B, H, NC, Q, generator=g) * 0.1 + 0.01).to(torch.bfloat16)
        return tuple(t.to(dev) for t in (x, cb, dA, Cm, prev, dt))

    def cpu(inp):
        from oracle import reference as ref

        return ref.ssd_chunk_scan(*inp, G)

    def sample(inp, rows):  # one chunk of batch 0, all heads
        x, cb, dA, Cm, prev, dt = inp
        return (x[:1, :Q], cb[:1, :1], dA[:1, :, :1], Cm[:1, :Q], prev[:1, :1], dt[:1, :, :1])

    def units(inp):  # bytes of the sample by the op's formula
        x, cb, dA, Cm, prev, dt = inp
        b, s, h, pp = x.shape
        tok = b * s * h
        return float(tok * pp * 2 + cb.numel() * 2 + tok * 4 + Cm.numel() * 2 + prev.numel() * 4
                     + tok * 2 + tok * pp * 4)

    return Workload(
        name="ssd_chunk_scan", metric="achieved HBM GB/s (SSDChunkScanFwdOp)", unit="GB/s",
        dtype="bf16",
        config={"workload": "SSDChunkScanFwdOp x (4, 2048, 80, 64) bf16, chunk 256, d_state "
                            "128, 1 group (manifest mamba2-2p7b-b4-s2k)"},
        make_inputs=make, build_op=SSDChunkScanFwdOp,
        run=lambda op, inp: op(*inp),
        work_per_step=lambda op: float(op.eval_roofline()[1]),
        kernel_regex="ssd_chunk_scan", cpu_fn=cpu, cpu_slice=sample, cpu_units=units,
    )


def _conv_dense() -> Workload:
    from tileops.ops.convolution import Conv1dBiasFwdOp

    N, CI, L, CO, K = 1, 80, 3000, 1280, 3

    def make(dev, seed):
        g = torch.Generator(device="cpu").manual_seed(seed)
        x = torch.randn(N, CI, L, generator=g).to(torch.float16)
        w = (torch.randn(CO, CI, K, generator=g) * 0.1).to(torch.float16)
        b = (torch.randn(CO, generator=g) * 0.1).to(torch.float16)
        return tuple(t.to(dev) for t in (x, w, b))

    def cpu(inp):
        from oracle import reference as ref

        return ref.conv1d(inp[0], inp[1], inp[2], 1, 0, 1, 1)

    def sample(inp, rows):  # a slice of the output channels
        co = max(8, min(CO, rows))
        return (inp[0], inp[1][:co], inp[2][:co])

    def units(inp):
        co = inp[1].shape[0]
        return float(2 * N * co * CI * (L - K + 1) * K)

    return Workload(
        name="conv1d_dense", unit="TFLOP/s", dtype="f16", bound="tensor",
        metric="achieved TFLOP/s (Conv1dBiasFwdOp, dense)",
        config={"workload": "Conv1dBiasFwdOp x (1, 80, 3000) f16, weight (1280, 80, 3), bias, "
                            "stride 1, no padding (manifest whisper-conv1-bias)"},
        make_inputs=make, build_op=lambda: Conv1dBiasFwdOp(),
        run=lambda op, inp: op(*inp), work_per_step=lambda op: float(op.eval_roofline()[0]),
        kernel_regex="conv1d_igemm", cpu_fn=cpu, cpu_slice=sample, cpu_units=units,
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
        g_ = torch.Generator(device="cpu").manual_seed(seed)
        q = F.normalize(torch.randn(1, TOTAL, H, DK, generator=g_), dim=-1).to(torch.bfloat16)
        k = F.normalize(torch.randn(1, TOTAL, H, DK, generator=g_), dim=-1).to(torch.bfloat16)
        v = torch.randn(1, TOTAL, H, DV, generator=g_).to(torch.bfloat16)
        g = F.logsigmoid(torch.randn(1, TOTAL, H, generator=g_)) / 16
        beta = torch.sigmoid(torch.randn(1, TOTAL, H, generator=g_))
        cu = torch.tensor(offsets, dtype=torch.int32)
        return tuple(t.to(dev) for t in (q, k, v, g, beta, cu))

    def cpu(inp):
        from oracle import reference as ref

        return ref.gdn_prefill_varlen(*inp[:5], inp[5])

    def sample(inp, rows):  # the first sequence's first tokens, one head
        t = max(64, min(offsets[1], rows * 4))
        return tuple(x[:1, :t, :1].contiguous() for x in inp[:5]) + (
            torch.tensor([0, t], dtype=torch.int32),)

    def units(inp):
        t = inp[0].shape[1]
        return float(t * (4 * 64 * DK + 6 * DK * DV + 3 * 64 * DV))

    return Workload(
        name="gdn_varlen", unit="TFLOP/s", dtype="bf16", bound="hbm", roof_unit="GB/s",
        roof_work_per_step=lambda op: float(op.eval_roofline()[1]),
        metric="achieved TFLOP/s (GatedDeltaNetPrefillFwdOp, packed cu_seqlens)",
        config={"workload": "GatedDeltaNetPrefillFwdOp packed: 32768 tokens (the BASELINE "
                            "token count) in 12 seeded ragged sequences, H=16 dk=dv=128, "
                            "chunk 64, same input distributions as the BASELINE config",
                "cu_seqlens": offsets},
        make_inputs=make,
        build_op=lambda: GatedDeltaNetPrefillFwdOp(1, TOTAL, H, DK, DV),
        run=lambda op, inp: op(*inp[:5], None, cu_seqlens=inp[5]),
        work_per_step=lambda op: float(op.eval_roofline()[0]),
        kernel_regex="gdn_", cpu_fn=cpu, cpu_slice=sample, cpu_units=units,
        launches_per_step=3,  # chunk index + prepare + scan
    )


def workloads() -> dict[str, Callable[[], Workload]]:
    table = {
        "fused_add_layer_norm": _faln,
        "gelu_and_mul": lambda: _gated(False),
        "gelu_tanh_and_mul": lambda: _gated(True),
        "causal_conv1d": lambda: _causal_conv(None),
        "causal_conv1d_silu": lambda: _causal_conv("silu"),
        "mha": lambda: _mha(False),
        "mha_causal": lambda: _mha(True),
        "gdn": _gdn,
        "gdn_varlen": _gdn_varlen,
        "gla_decode": _gla,
        "ssd_chunk_scan": _ssd,
        "conv1d_dense": _conv_dense,
    }
    for kind in ("hardswish", "hardsigmoid", "clamp_scalar", "isnan", "isinf", "isfinite",
                 "bitwise_not"):
        table[kind] = (lambda k: (lambda: _unary(k)))(kind)
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
    """DRAM bytes per launch of the op's dominant kernel from the committed ncu summary."""
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
            self._thread = threading.Thread(target=self._loop, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join()
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


def gather_outputs(outs, world: int, device, reps: int = 5):
    """Reassemble every rank's output shards on every rank: one
    ``all_gather_into_tensor`` per output tensor (NCCL over NVLink on GPUs,
    gloo on CPU ranks).  It moves results only -- no op needs data from
    another rank -- so it is timed apart from the op: the mean of ``reps``
    rounds, the max over ranks.  Returns (summary, gathered tensors)."""
    import torch.distributed as dist

    flats = [o.contiguous().view(-1) for o in outs]
    fulls = [torch.empty(world * f.numel(), dtype=f.dtype, device=f.device) for f in flats]

    def one_round():
        for full, flat in zip(fulls, flats):
            dist.all_gather_into_tensor(full, flat)

    one_round()  # warm-up; its result is what the caller checks
    barrier(world, device)
    if device.type == "cuda":
        torch.cuda.synchronize(device)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(torch.cuda.current_stream(device))
        for _ in range(reps):
            one_round()
        e1.record(torch.cuda.current_stream(device))
        torch.cuda.synchronize(device)
        ms = e0.elapsed_time(e1) / reps
    else:
        t0 = time.perf_counter()
        for _ in range(reps):
            one_round()
        ms = (time.perf_counter() - t0) * 1e3 / reps
    ms = max_over_ranks(ms, world, device)
    per_rank = sum(f.numel() * f.element_size() for f in flats)
    total = world * per_rank
    summary = {
        "collective": "all_gather_into_tensor (output reassembly only)",
        "outputs": len(flats), "bytes_per_rank": per_rank, "bytes_total": total,
        "bytes_received_per_rank": (world - 1) * per_rank, "ms": ms,
        "algbw_GBps": total / (ms * 1e-3) / 1e9,
        "busbw_GBps": (world - 1) / world * total / (ms * 1e-3) / 1e9,
    }
    return summary, fulls


def whole_job_value(work_per_step: float, steps: int, total_ms: float, world: int,
                    unit: str) -> float:
    """Weak scaling: every rank ran ``steps`` steps of ``work_per_step`` units;
    ``total_ms`` is the slowest rank's timed region."""
    scale = 1e9 if unit == "GB/s" else 1e12
    return world * work_per_step * steps / (total_ms * 1e-3) / scale


# ---------------------------------------------------------------- our arm
def time_cpu_baseline(wl: Workload, budget_s: float = 8.0) -> dict:
    """The oracle (the reference's torch CPU ref program) on a bounded sample."""
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    full = wl.make_inputs(torch.device("cpu"), 1235)
    rows = 256
    sample = wl.cpu_slice(full, rows)
    wl.cpu_fn(sample)  # warm-up
    times = []
    t_end = time.perf_counter() + budget_s
    while time.perf_counter() < t_end or len(times) < 3:
        t0 = time.perf_counter()
        wl.cpu_fn(sample)
        times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    units = wl.cpu_units(sample)
    value = units / med / (1e9 if wl.unit == "GB/s" else 1e12)
    desc = ", ".join(f"{tuple(t.shape)}" for t in sample if isinstance(t, torch.Tensor))
    return {"value": value, "unit": wl.unit, "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"oracle on inputs {desc}, median of {len(times)} reps ({med*1e3:.2f} ms)",
            "cpu_count": os.cpu_count()}


def run_ours(args, wl: Workload) -> Optional[dict]:
    rank, local_rank, world = dist_env()
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=device)
    op = wl.build_op()
    probe = wl.make_inputs(device, 1235 + rank)
    set_bytes = sum(t.numel() * t.element_size() for t in probe if isinstance(t, torch.Tensor))
    out = wl.run(op, probe)
    outs = out if isinstance(out, (tuple, list)) else (out,)
    set_bytes += sum(t.numel() * t.element_size() for t in outs)
    del out, outs
    n_sets = max(2, min(32, -(-3 * L2_BYTES // max(set_bytes, 1)) + 1))
    sets = [probe] + [wl.make_inputs(device, 1235 + rank + 1000 * i) for i in range(1, n_sets)]
    work = wl.work_per_step(op)
    stream = torch.cuda.current_stream(device)

    for i in range(args.warmup):
        wl.run(op, sets[i % n_sets])
    torch.cuda.synchronize(device)

    # Graph mode: a CUDA graph holds R consecutive op calls (validation,
    # output allocation, the library's launches) over the rotating input
    # sets, each call with outputs of its own; K steps replay it K // R times
    # (plus a graph of the K % R remaining calls).  Eager mode calls the op
    # K times from Python.
    out_bytes = max(1, set_bytes - sum(t.numel() * t.element_size() for t in probe
                                       if isinstance(t, torch.Tensor)))
    per_graph = max(1, min(64, (8 << 30) // out_bytes) // n_sets) * n_sets
    per_graph = min(per_graph, args.steps)

    def capture(n):
        graph = torch.cuda.CUDAGraph()
        keep = []
        with torch.cuda.graph(graph):
            for i in range(n):
                keep.append(wl.run(op, sets[i % n_sets]))
        del keep
        return graph

    if args.graph:
        g_main = capture(per_graph)
        rem = args.steps % per_graph
        g_rem = capture(rem) if rem else None
        chunks = [(g_main.replay, per_graph)] * (args.steps // per_graph)
        if g_rem is not None:
            chunks.append((g_rem.replay, rem))
        for _ in range(max(1, -(-args.warmup // per_graph))):
            g_main.replay()
        torch.cuda.synchronize(device)
    else:
        chunks = [((lambda inp=sets[i % n_sets]: wl.run(op, inp)), 1) for i in range(args.steps)]

    starts = [torch.cuda.Event(enable_timing=True) for _ in chunks]
    ends = [torch.cuda.Event(enable_timing=True) for _ in chunks]
    sampler = ClockSampler(local_rank)
    barrier(world, device)
    torch.cuda.synchronize(device)
    with sampler:
        for i, (fn, _) in enumerate(chunks):
            starts[i].record(stream)
            fn()
            ends[i].record(stream)
        torch.cuda.synchronize(device)
    barrier(world, device)
    total_ms = starts[0].elapsed_time(ends[-1])
    # Mean step time inside the timed calls (excludes host gaps between them).
    per_launch_ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends)) / args.steps
    chunk_steps = [n for _, n in chunks]
    del chunks
    if args.graph:
        del g_main, g_rem
    total_ms = max_over_ranks(total_ms, world, device)
    per_launch_ms = max_over_ranks(per_launch_ms, world, device)

    # End to end through the public API with pinned host buffers.
    host_in = [t.cpu().pin_memory() if isinstance(t, torch.Tensor) else t for t in sets[0]]
    out = wl.run(op, sets[0])
    outs = out if isinstance(out, (tuple, list)) else (out,)
    host_out = [torch.empty(o.shape, dtype=o.dtype, pin_memory=True) for o in outs]
    h2d = sum(t.numel() * t.element_size() for t in host_in if isinstance(t, torch.Tensor))
    d2h = sum(t.numel() * t.element_size() for t in host_out)
    e2e_steps = max(3, min(args.steps, 30))

    def e2e_step():
        dev_in = [t.to(device, non_blocking=True) if isinstance(t, torch.Tensor) else t
                  for t in host_in]
        res = wl.run(op, tuple(dev_in))
        res = res if isinstance(res, (tuple, list)) else (res,)
        for h, d in zip(host_out, res):
            h.copy_(d, non_blocking=True)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize(device)
    barrier(world, device)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize(device)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / e2e_steps, world, device)
    barrier(world, device)

    gather = None
    if args.gather and world > 1:
        res = wl.run(op, sets[0])
        res = res if isinstance(res, (tuple, list)) else (res,)
        gather, fulls = gather_outputs(res, world, device)
        gather["op_plus_gather_ms"] = per_launch_ms + gather["ms"]
        del res, fulls
        barrier(world, device)

    scale = 1e9 if wl.unit == "GB/s" else 1e12
    value = whole_job_value(work, args.steps, total_ms, world, wl.unit)
    roof_unit = wl.roof_unit or wl.unit
    roof_work = wl.roof_work_per_step(op) if wl.roof_work_per_step else work
    roof_scale = 1e9 if roof_unit == "GB/s" else 1e12
    achieved = roof_work / (per_launch_ms * 1e-3) / roof_scale
    peaks, peak_kind = load_peaks()
    if roof_unit == "GB/s":
        peak = float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
        peak_unit = "GB/s"
    else:
        peak = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
        peak_unit = "TFLOP/s"
    clocks = sampler.summary()
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    if rank != 0:
        return None
    line = {
        "metric": wl.metric, "value": value, "unit": wl.unit, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": total_ms / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": wl.dtype,
        "data": "synthetic (seeded torch.randn of the BASELINE shapes)",
        "config": {**wl.config, "parallelism": f"independent batch per GPU x{world}",
                   "l2": f"rotating {n_sets} input/output sets "
                         f"({n_sets * set_bytes / 2**20:.0f} MiB) > 126 MB L2",
                   "timing": (f"CUDA-graph replays of {chunk_steps[0]} op calls each, "
                              "CUDA events around each replay" if args.graph else
                              "eager op calls, CUDA events per step")},
        "roofline": {"bound": wl.bound, "achieved": achieved, "peak": peak, "unit": peak_unit,
                     "frac": achieved / peak, "traffic": load_traffic(wl.name),
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json)" if peak_kind ==
                     "measured" else "fallback", "per_launch_ms": per_launch_ms,
                     "algorithmic_per_launch": roof_work},
        "e2e": {"value": whole_job_value(work, 1, e2e_ms, world, wl.unit), "unit": wl.unit,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms,
                "api": f"{type(op).__name__}.__call__ with pinned host buffers"},
        "gpu_launches": args.steps * wl.launches_per_step,
        "clocks": clocks,
    }
    if gather is not None:
        line["gather"] = gather
    if world == 1 and not args.no_cpu_baseline and wl.cpu_fn is not None:
        line["cpu_baseline"] = time_cpu_baseline(wl)
    return line


# ----------------------------------------------------------- reference arm
def run_reference(args, wl: Workload) -> Optional[dict]:
    rank, _, world = dist_env()
    if rank != 0:
        return None
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    full = wl.make_inputs(torch.device("cpu"), 1235)
    rows = args.ref_rows
    sample = wl.cpu_slice(full, rows)
    for _ in range(args.warmup):
        wl.cpu_fn(sample)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        wl.cpu_fn(sample)
    sec = (time.perf_counter() - t0) / args.steps
    scale = 1e9 if wl.unit == "GB/s" else 1e12
    value = wl.cpu_units(sample) / sec / scale
    desc = ", ".join(f"{tuple(t.shape)}" for t in sample if isinstance(t, torch.Tensor))
    return {
        "impl": "reference", "metric": wl.metric, "value": value, "unit": wl.unit,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": sec * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": wl.dtype,
        "data": "synthetic (seeded torch.randn of the BASELINE shapes)",
        "config": {**wl.config, "parallelism": "host CPU, rank 0 only"},
        "cpu_baseline": {"value": value, "unit": wl.unit, "cores": torch.get_num_threads(),
                         "kind": "port",
                         "sample": f"reference torch CPU ref program (restated in oracle/) on "
                                   f"inputs {desc} per step"},
        "e2e": {"value": value, "unit": wl.unit, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def main() -> None:
    ap = argparse.ArgumentParser(description="B200 TileOPs hot-path benchmark")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--op", default="fused_add_layer_norm")
    ap.add_argument("--ref-rows", type=int, default=256,
                    help="rows of the batch the CPU reference processes per step")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-graph", dest="graph", action="store_false",
                    help="time eager op calls instead of CUDA-graph replays")
    ap.add_argument("--gather", action="store_true",
                    help="N > 1: also time reassembling every rank's outputs on every rank "
                         "(all_gather_into_tensor; reported under 'gather', not in 'value')")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    table = workloads()
    if args.op not in table:
        raise SystemExit(f"unknown --op {args.op}; choose from {sorted(table)}")
    wl = table[args.op]()
    line = run_reference(args, wl) if args.impl == "reference" else run_ours(args, wl)
    if line is not None:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
