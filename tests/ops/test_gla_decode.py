"""GLADecodeOp against the GLA decode golden.

The reference test (examples/TileOPs/tests/ops/test_gla_decode.py:26-69)
compares o and new_state with the fp32 golden at its per-dtype tolerance
(fp16 2e-3, bf16 2e-2, fp32 1e-4, gla_decode_tolerance); the same cases run
here, plus the committed golden fixtures, a DV that is not a multiple of a
16-byte packet (element path), many-head shapes and determinism.  The
constructor-level checks (default scale, eval_roofline) need no GPU.
"""

import pytest
import torch

from oracle import reference as ref
from tests.golden.load import load, names
from tileops.ops.linear_attention import GLADecodeOp
from tileops.workloads.linear_attention import GLADecodeWorkload, gla_decode_tolerance

_F16, _BF16, _F32 = torch.float16, torch.bfloat16, torch.float32

_CASES = [
    (2, 4, 64, 64, _F16, -1.0),
    (2, 4, 64, 64, _BF16, -1.0),
    (1, 8, 128, 128, _BF16, -1.0),
    (1, 32, 128, 128, _BF16, -1.0),
    (8, 32, 128, 128, _BF16, -1.0),
    (1, 2, 32, 16, _F32, -1.0),
    (2, 3, 16, 16, _F16, -1.0),
    (1, 4, 128, 64, _F16, -1.0),
    (2, 3, 64, 64, _BF16, 0.25),
    (3, 5, 40, 12, _BF16, -1.0),    # DV not a packet multiple: element path
    (64, 64, 64, 128, _F16, -1.0),  # many (b, h): no column slicing
    (1, 1, 256, 1024, _F32, 0.5),   # one (b, h): many column slices
]


def _check(op, q, k, v, gk, state, scale, dtype):
    o, ns = op(q, k, v, gk, state)
    assert o.dtype == dtype and ns.dtype == dtype
    ref_o, ref_ns = ref.gla_decode(q, k, v, gk, state, scale)
    tol = gla_decode_tolerance(dtype)
    torch.testing.assert_close(o.cpu().float(), ref_o, **tol)
    torch.testing.assert_close(ns.cpu().float(), ref_ns, **tol)
    return o, ns


@pytest.mark.gpu
@pytest.mark.parametrize("B, H, DK, DV, dtype, scale", _CASES)
def test_gla_decode(B, H, DK, DV, dtype, scale):
    torch.manual_seed(1235)
    wl = GLADecodeWorkload(B, H, DK, DV, dtype, scale)
    q, k, v, gk, state = wl.gen_inputs()
    op = GLADecodeOp(B, H, DK, DV, scale=scale, dtype=dtype)
    _check(op, q, k, v, gk, state, op.kernel.scale, dtype)


@pytest.mark.gpu
@pytest.mark.parametrize("name", names("gla_decode_"))
def test_gla_decode_golden_fixtures(name):
    case = load(name)
    i, m = case["inputs"], case["meta"]
    B, H, DK = i["q"].shape
    DV = i["v"].shape[-1]
    dtype = i["q"].dtype
    op = GLADecodeOp(B, H, DK, DV, scale=m["scale_arg"], dtype=dtype)
    assert op.kernel.scale == pytest.approx(m["scale"])
    o, ns = op(*(i[n].cuda() for n in ("q", "k", "v", "gk", "state")))
    tol = gla_decode_tolerance(dtype)
    torch.testing.assert_close(o.cpu().float(), case["outputs"]["o"], **tol)
    torch.testing.assert_close(ns.cpu().float(), case["outputs"]["new_state"], **tol)


@pytest.mark.gpu
def test_gla_decode_deterministic_and_new_state_rounding():
    wl = GLADecodeWorkload(2, 8, 128, 128, _BF16)
    q, k, v, gk, state = wl.gen_inputs()
    op = GLADecodeOp(2, 8, 128, 128, dtype=_BF16)
    o0, ns0 = op(q, k, v, gk, state)
    o1, ns1 = op(q, k, v, gk, state)
    assert torch.equal(o0, o1) and torch.equal(ns0, ns1)
    # new_state is the fp32 update rounded once: within half a bf16 ulp of it
    _, ref_ns = ref.gla_decode(q, k, v, gk, state, op.kernel.scale)
    diff = (ns0.cpu().float() - ref_ns).abs()
    assert bool((diff <= ref_ns.abs() * 2.0 ** -8 + 1e-6).all())


@pytest.mark.gpu
def test_gla_decode_rejects_bad_inputs():
    wl = GLADecodeWorkload(1, 2, 64, 64, _BF16)
    q, k, v, gk, state = wl.gen_inputs()
    op = GLADecodeOp(1, 2, 64, 64, dtype=_BF16)
    with pytest.raises(ValueError, match="state.shape"):
        op(q, k, v, gk, state[:, :, :32])
    with pytest.raises(ValueError, match="q.dtype"):
        op(q.half(), k, v, gk, state)
    with pytest.raises(ValueError, match="must be a cuda tensor"):
        op(q.cpu(), k, v, gk, state)


def test_gla_decode_default_scale():
    """A non-positive scale resolves to ``DK ** -0.5`` (reference test :72-76)."""
    op = GLADecodeOp(1, 2, 64, 64, scale=-1.0, dtype=torch.float16)
    assert op.kernel.scale == pytest.approx(64 ** -0.5)
    assert GLADecodeOp(1, 2, 64, 64, scale=0.25).kernel.scale == 0.25


def test_gla_decode_eval_roofline():
    B, H, DK, DV = 1, 8, 128, 128
    op = GLADecodeOp(B, H, DK, DV, dtype=torch.bfloat16)
    flops, nbytes = op.eval_roofline()
    assert flops == B * H * (5 * DK * DV + DK + DV)
    assert nbytes == B * H * (3 * DK + 2 * DV + 2 * DK * DV) * 2


def test_gla_decode_rejects_unsupported_dtype():
    with pytest.raises(ValueError, match="only supports dtypes"):
        GLADecodeOp(1, 2, 64, 64, dtype=torch.int32)
