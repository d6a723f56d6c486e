"""GPU parity of the flat elementwise ops against the oracle and the golden fixtures.

Ported from the reference tests (TO/tests/ops/test_hardswish.py,
test_hardsigmoid.py, test_clamp_scalar.py, test_clamp_min.py, test_isnan.py,
test_isinf.py, test_isfinite.py, test_bitwise_not.py): same parameter sweeps
and tolerances (fp32 1e-5; fp16 1e-3; bf16 1.6e-2; exact for predicates and
bitwise ops), with ref_program = the CPU oracle.  Added: the reference-output
fixtures with IEEE corner values, ragged / misaligned sizes (scalar path and
vector tails), and BASELINE's 256M-element shape checked on a strided sample
(the ops are elementwise, so sampled positions are exact checks).
"""

import pytest
import torch

from oracle import reference as ref
from tests.golden.load import load, names
from tileops.ops.elementwise import (
    BitwiseNotFwdOp,
    ClampMinFwdOp,
    ClampScalarFwdOp,
    HardsigmoidFwdOp,
    HardswishFwdOp,
    IsfiniteFwdOp,
    IsinfFwdOp,
    IsnanFwdOp,
)
from tileops.testing.test_base import TestBase
from tileops.workloads.elementwise import (
    BitwiseNotWorkload,
    IsfiniteWorkload,
    IsinfWorkload,
    IsnanWorkload,
)
from tileops.workloads.workload_base import RandnWorkload

pytestmark = pytest.mark.gpu

TOL = {torch.float32: (1e-5, 1e-5), torch.float16: (1e-3, 1e-3), torch.bfloat16: (1.6e-2, 1.6e-2)}
FLOATS = [torch.float32, torch.float16, torch.bfloat16]
SIZES = [
    pytest.param(1_048_576, torch.float32, marks=pytest.mark.smoke),
    pytest.param(1_048_576, torch.float16, marks=pytest.mark.smoke),
    pytest.param(1_048_576, torch.bfloat16, marks=pytest.mark.smoke),
    pytest.param(4_000_000, torch.float16, marks=pytest.mark.full),
    pytest.param(4_000_000, torch.bfloat16, marks=pytest.mark.full),
]


class _UnaryTest(RandnWorkload, TestBase):
    def __init__(self, n, dtype, fn):
        super().__init__((n,), dtype)
        self.fn = fn

    def ref_program(self, x):
        return self.fn(x)


@pytest.mark.parametrize("n_total, dtype", SIZES)
@pytest.mark.parametrize("op_cls,fn", [(HardswishFwdOp, ref.hardswish),
                                       (HardsigmoidFwdOp, ref.hardsigmoid)])
def test_activation_op(op_cls, fn, n_total, dtype):
    test = _UnaryTest(n_total, dtype, fn)
    atol, rtol = TOL[dtype]
    test.check(op_cls(N_total=n_total, dtype=dtype), *test.gen_inputs(), atol=atol, rtol=rtol)


@pytest.mark.parametrize("n_total, dtype", SIZES)
def test_clamp_scalar_op(n_total, dtype):
    test = _UnaryTest(n_total, dtype, lambda x: ref.clamp_scalar(x, -0.5, 0.5))
    atol, rtol = TOL[dtype]
    op = ClampScalarFwdOp(N_total=n_total, dtype=dtype, min=-0.5, max=0.5)
    test.check(op, *test.gen_inputs(), atol=atol, rtol=rtol)


@pytest.mark.parametrize("min_val, max_val", [(-0.5, 0.5), (None, 0.5), (-0.5, None)])
def test_clamp_scalar_param_names(min_val, max_val):
    test = _UnaryTest(1024, torch.float32, lambda x: ref.clamp_scalar(x, min_val, max_val))
    test.check(ClampScalarFwdOp(N_total=1024, dtype=torch.float32, min=min_val, max=max_val),
               *test.gen_inputs())


@pytest.mark.parametrize("dtype", FLOATS)
def test_clamp_min_op(dtype):
    test = _UnaryTest(1_048_576, dtype, lambda x: ref.clamp_min(x, -0.5))
    atol, rtol = TOL[dtype]
    test.check(ClampMinFwdOp(N_total=1_048_576, dtype=dtype, min=-0.5), *test.gen_inputs(),
               atol=atol, rtol=rtol)


def _pred_cls(name):
    return {"isnan": (IsnanFwdOp, IsnanWorkload, ref.isnan),
            "isinf": (IsinfFwdOp, IsinfWorkload, ref.isinf),
            "isfinite": (IsfiniteFwdOp, IsfiniteWorkload, ref.isfinite)}[name]


@pytest.mark.parametrize("n_total, dtype", SIZES)
@pytest.mark.parametrize("pred", ["isnan", "isinf", "isfinite"])
def test_predicate_op(pred, n_total, dtype):
    op_cls, wl_cls, fn = _pred_cls(pred)

    class T(wl_cls, TestBase):
        def ref_program(self, x):
            return fn(x)

    test = T((n_total,), dtype)
    test.check(op_cls(N_total=n_total, dtype=dtype), *test.gen_inputs(), atol=0.0, rtol=0.0)


def test_isnan_output_dtype_and_values():
    n = 4096
    op = IsnanFwdOp(N_total=n, dtype=torch.float32)
    x = torch.randn(n, device="cuda")
    x[: n // 2] = float("nan")
    y = op(x)
    assert y.dtype == torch.bool and tuple(y.shape) == (n,)
    assert bool(y[: n // 2].all()) and not bool(y[n // 2 :].any())


BITWISE = [
    pytest.param(1_048_576, torch.int32, marks=pytest.mark.smoke),
    pytest.param(1_048_576, torch.int64, marks=pytest.mark.smoke),
    pytest.param(1_048_576, torch.bool, marks=pytest.mark.smoke),
    pytest.param(1_048_576, torch.uint8, marks=pytest.mark.smoke),
    pytest.param(1_048_576, torch.int8, marks=pytest.mark.smoke),
    pytest.param(1_048_576, torch.int16, marks=pytest.mark.smoke),
    pytest.param(4_000_000, torch.int32, marks=pytest.mark.full),
    pytest.param(4_000_000, torch.int64, marks=pytest.mark.full),
]


@pytest.mark.parametrize("n_total, dtype", BITWISE)
def test_bitwise_not_op(n_total, dtype):
    class T(BitwiseNotWorkload, TestBase):
        def ref_program(self, x):
            return ref.bitwise_not(x)

    test = T((n_total,), dtype)
    test.check(BitwiseNotFwdOp(N_total=n_total, dtype=dtype), *test.gen_inputs(), atol=0.0,
               rtol=0.0)


# ------------------------------------------------------- golden fixtures
def _run_fixture_op(name, x):
    kind = name.rsplit("_", 1)[0]
    n = x.numel()
    if kind == "hardswish":
        return HardswishFwdOp(n, x.dtype)(x)
    if kind == "hardsigmoid":
        return HardsigmoidFwdOp(n, x.dtype)(x)
    if kind.startswith("clamp_scalar"):
        m = load(name)["meta"]
        return ClampScalarFwdOp(n, x.dtype, min=m["min"], max=m["max"])(x)
    if kind == "clamp_min":
        return ClampMinFwdOp(n, x.dtype, min=load(name)["meta"]["min"])(x)
    if kind in ("isnan", "isinf", "isfinite"):
        return _pred_cls(kind)[0](n, x.dtype)(x)
    if kind == "bitwise_not":
        return BitwiseNotFwdOp(n, x.dtype)(x)
    raise KeyError(name)


FIXTURES = (names("hardswish_") + names("hardsigmoid_") + names("clamp_") + names("isnan_")
            + names("isinf_") + names("isfinite_") + names("bitwise_not_"))


@pytest.mark.parametrize("name", FIXTURES)
def test_reference_fixture(name):
    case = load(name)
    x = case["inputs"]["x"].cuda()
    y = _run_fixture_op(name, x).cpu()
    expect = case["outputs"]["y"]
    assert y.dtype == expect.dtype and y.shape == expect.shape
    if expect.dtype.is_floating_point:
        atol, rtol = TOL[expect.dtype]
        torch.testing.assert_close(y, expect, atol=atol, rtol=rtol, equal_nan=True)
        # NaN / Inf positions must agree exactly.
        assert torch.equal(torch.isnan(y), torch.isnan(expect))
        assert torch.equal(torch.isinf(y), torch.isinf(expect))
    else:
        assert torch.equal(y, expect)


# ------------------------------------------- ragged sizes, misaligned views
@pytest.mark.parametrize("n", [1, 7, 15, 16, 17, 4097, 65_537])
@pytest.mark.parametrize("dtype", FLOATS)
@pytest.mark.parametrize("offset", [0, 1])
def test_ragged_and_misaligned(n, dtype, offset):
    base = torch.randn(n + offset, device="cuda", dtype=dtype)
    base[::3] = float("nan")
    base[1::5] = float("inf")
    base[2::7] = float("-inf")
    x = base[offset:]  # offset 1 breaks 16-byte alignment -> scalar kernel
    atol, rtol = TOL[dtype]
    torch.testing.assert_close(HardswishFwdOp(n, dtype)(x).cpu(), ref.hardswish(x),
                               atol=atol, rtol=rtol, equal_nan=True)
    torch.testing.assert_close(ClampScalarFwdOp(n, dtype, min=-0.3, max=0.7)(x).cpu(),
                               ref.clamp_scalar(x, -0.3, 0.7), atol=atol, rtol=rtol,
                               equal_nan=True)
    for pred in ("isnan", "isinf", "isfinite"):
        op_cls, _, fn = _pred_cls(pred)
        assert torch.equal(op_cls(n, dtype)(x).cpu(), fn(x))


@pytest.mark.parametrize("n", [1, 3, 17, 4099])
@pytest.mark.parametrize("dtype", [torch.bool, torch.int8, torch.int16, torch.int32, torch.int64])
def test_bitwise_not_ragged_misaligned(n, dtype):
    (base,) = BitwiseNotWorkload((n + 1,), dtype).gen_inputs()
    for x in (base[:n], base[1:]):
        assert torch.equal(BitwiseNotFwdOp(n, dtype)(x).cpu(), ref.bitwise_not(x))


def test_inplace_preserves_identity():
    x = torch.randn(1000, device="cuda", dtype=torch.bfloat16)
    expect = ref.hardswish(x)
    y = HardswishFwdOp(1000, torch.bfloat16, inplace=True)(x)
    assert y is x
    torch.testing.assert_close(x.cpu(), expect, atol=1.6e-2, rtol=1.6e-2)


def test_shape_is_preserved():
    x = torch.randn(32, 96, 7, 7, device="cuda", dtype=torch.float16)
    y = HardsigmoidFwdOp(x.numel(), torch.float16)(x)
    assert y.shape == x.shape
    torch.testing.assert_close(y.cpu(), ref.hardsigmoid(x), atol=1e-3, rtol=1e-3)


# ------------------------------------------------ BASELINE size: 16384^2
@pytest.mark.full
def test_baseline_size_sampled():
    shape = (16384, 16384)
    n = shape[0] * shape[1]
    x = torch.randn(shape, device="cuda", dtype=torch.bfloat16)
    x.view(-1)[::1001] = float("nan")
    idx = torch.arange(0, n, 9973, device="cuda")  # strided sample over the whole range
    xs = x.view(-1)[idx]
    y = HardswishFwdOp(n, torch.bfloat16)(x).view(-1)[idx]
    torch.testing.assert_close(y.cpu(), ref.hardswish(xs), atol=1.6e-2, rtol=1.6e-2,
                               equal_nan=True)
    assert torch.equal(IsnanFwdOp(n, torch.bfloat16)(x).view(-1)[idx].cpu(), ref.isnan(xs))
    c = ClampScalarFwdOp(n, torch.bfloat16, min=-0.5, max=0.5)(x).view(-1)[idx]
    torch.testing.assert_close(c.cpu(), ref.clamp_scalar(xs, -0.5, 0.5), atol=0, rtol=0,
                               equal_nan=True)
    del x
    xi = torch.randint(-128, 128, shape, device="cuda", dtype=torch.int32)
    yi = BitwiseNotFwdOp(n, torch.int32)(xi)
    assert torch.equal(yi, ~xi)  # device-side exact check of every element


# --------------------------------- every 16-bit encoding, bit for bit
def _all_encodings(dtype):
    return torch.arange(-32768, 32768, dtype=torch.int32).to(torch.int16).view(dtype)


def _same_bits(y, expect):
    """Equal encodings, any NaN matching any NaN (payloads are not part of the contract)."""
    nan_y, nan_e = torch.isnan(y), torch.isnan(expect)
    assert torch.equal(nan_y, nan_e)
    keep = ~nan_e
    assert torch.equal(y[keep].view(torch.int16), expect[keep].view(torch.int16))


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_all_16bit_inputs_bit_exact(dtype):
    """Hardswish, hardsigmoid and clamp over all 65536 inputs equal the fp32
    reference rounded once (the kernels divide by 6 as a multiply by RN(1/6)
    on these types, which this pins)."""
    x = _all_encodings(dtype)
    xd = x.cuda()
    n = x.numel()
    _same_bits(HardswishFwdOp(n, dtype)(xd).cpu(), ref.hardswish(x))
    _same_bits(HardsigmoidFwdOp(n, dtype)(xd).cpu(), ref.hardsigmoid(x))
    _same_bits(ClampScalarFwdOp(n, dtype, min=-0.5, max=0.5)(xd).cpu(),
               ref.clamp_scalar(x, -0.5, 0.5))
    _same_bits(ClampScalarFwdOp(n, dtype, min=None, max=2.0)(xd).cpu(),
               ref.clamp_scalar(x, None, 2.0))
    _same_bits(ClampMinFwdOp(n, dtype, min=-1.0)(xd).cpu(), ref.clamp_scalar(x, -1.0, None))


def test_clamp_nan_bound_propagates():
    x = torch.randn(4096, device="cuda")
    y = ClampScalarFwdOp(4096, torch.float32, min=float("nan"), max=1.0)(x).cpu()
    expect = torch.clamp(x.cpu(), min=float("nan"), max=1.0)
    assert torch.equal(torch.isnan(y), torch.isnan(expect))
