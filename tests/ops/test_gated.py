"""GPU parity of GeluAndMulFwdOp / GeluTanhAndMulFwdOp.

Ported from TO/tests/ops/test_gelu_and_mul.py and test_gelu_tanh_and_mul.py
(params: smoke (16, 128) x 3 dtypes; full (2048, 14336) fp16/bf16; decode
(1, 14336); tolerances fp32 1e-5, fp16 1e-2, bf16 1.6e-2), with the oracle as
ref_program.  Added: the reference-output fixtures (with IEEE corner gates
and values), widths that are not a multiple of the 16-byte packet (scalar
path), and BASELINE's (4096, 11008) bf16 config compared in full.
"""

import pytest
import torch

from oracle import reference as ref
from tests.golden.load import load, names
from tileops.ops.elementwise import GeluAndMulFwdOp, GeluTanhAndMulFwdOp
from tileops.testing.test_base import TestBase
from tileops.workloads.elementwise import GatedWorkload

pytestmark = pytest.mark.gpu

TOL = {torch.float32: (1e-5, 1e-5), torch.float16: (1e-2, 1e-2), torch.bfloat16: (1.6e-2, 1.6e-2)}
OPS = [(GeluAndMulFwdOp, ref.gelu_and_mul), (GeluTanhAndMulFwdOp, ref.gelu_tanh_and_mul)]
PARAMS = [
    pytest.param(16, 128, torch.float32, marks=pytest.mark.smoke),
    pytest.param(16, 128, torch.float16, marks=pytest.mark.smoke),
    pytest.param(16, 128, torch.bfloat16, marks=pytest.mark.smoke),
    pytest.param(2048, 14336, torch.float16, marks=pytest.mark.full),
    pytest.param(2048, 14336, torch.bfloat16, marks=pytest.mark.full),
    pytest.param(1, 14336, torch.bfloat16, marks=pytest.mark.full),
    pytest.param(4096, 11008, torch.bfloat16, marks=pytest.mark.full),  # BASELINE config
]


class GatedTest(GatedWorkload, TestBase):
    def __init__(self, M, N, dtype, fn):
        super().__init__(M, N, dtype)
        self.fn = fn

    def ref_program(self, x):
        return self.fn(x)


@pytest.mark.parametrize("M, N, dtype", PARAMS)
@pytest.mark.parametrize("op_cls,fn", OPS)
def test_gated_op(op_cls, fn, M, N, dtype):
    test = GatedTest(M, N, dtype, fn)
    atol, rtol = TOL[dtype]
    test.check(op_cls(M=M, N=N, dtype=dtype), *test.gen_inputs(), atol=atol, rtol=rtol)


@pytest.mark.parametrize("name", names("gelu_and_mul_") + names("gelu_tanh_and_mul_"))
def test_reference_fixture(name):
    case = load(name)
    x = case["inputs"]["x"].cuda()
    M, N = x.shape[0], x.shape[1] // 2
    op_cls = GeluTanhAndMulFwdOp if name.startswith("gelu_tanh") else GeluAndMulFwdOp
    y = op_cls(M, N, x.dtype)(x).cpu()
    expect = case["outputs"]["y"]
    atol, rtol = TOL[x.dtype]
    torch.testing.assert_close(y, expect, atol=atol, rtol=rtol, equal_nan=True)
    assert torch.equal(torch.isnan(y), torch.isnan(expect))


@pytest.mark.parametrize("N", [1, 3, 7, 9, 127, 1001])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("op_cls,fn", OPS)
def test_ragged_width(op_cls, fn, N, dtype):
    x = torch.randn(5, 2 * N, device="cuda", dtype=dtype)
    atol, rtol = TOL[dtype]
    torch.testing.assert_close(op_cls(5, N, dtype)(x).cpu(), fn(x), atol=atol, rtol=rtol)


def test_misaligned_input_view():
    base = torch.randn(4 * 256 + 1, device="cuda", dtype=torch.bfloat16)
    x = base[1:].view(4, 256)  # 2-byte offset -> scalar path
    torch.testing.assert_close(GeluAndMulFwdOp(4, 128, torch.bfloat16)(x).cpu(),
                               ref.gelu_and_mul(x), atol=1.6e-2, rtol=1.6e-2)


def test_empty_rows():
    x = torch.empty(0, 16, device="cuda", dtype=torch.float16)
    assert GeluAndMulFwdOp(0, 8, torch.float16)(x).shape == (0, 8)


@pytest.mark.parametrize("op_cls", [GeluAndMulFwdOp, GeluTanhAndMulFwdOp])
def test_activation_accuracy_dense_grid(op_cls):
    """The kernels evaluate erf by Abramowitz & Stegun 7.1.26 (|error| <= 1.5e-7)
    and tanh as 1 - 2 / (1 + exp(2u)); against fp64 the GELU error must stay
    below 0.5 * |g| * 3e-7 (approximation bound plus the approximate reciprocal
    and exp2), i.e. 2e-6 on [-12, 12], and the IEEE limits must hold."""
    g = torch.linspace(-12.0, 12.0, 200_001, dtype=torch.float64)
    g = torch.cat([g, torch.tensor([0.0, -0.0, 1e-30, -1e-30, float("inf"), float("-inf"),
                                    float("nan")], dtype=torch.float64)])
    n = g.numel()
    x = torch.cat([g.float(), torch.ones(n)]).reshape(1, 2 * n).cuda()  # gate | value = 1
    y = op_cls(1, n, torch.float32)(x).cpu().double()[0]
    g32 = g.float().double()
    if op_cls is GeluAndMulFwdOp:
        exact = 0.5 * g32 * (1.0 + torch.erf(g32 / 2**0.5))
    else:
        exact = 0.5 * g32 * (1.0 + torch.tanh((2 / torch.pi) ** 0.5 * (g32 + 0.044715 * g32**3)))
    finite = torch.isfinite(g32)
    err = (y[finite] - exact[finite]).abs()
    assert float(err.max()) <= 2e-6, float(err.max())
    assert y[-3] == float("inf") and torch.isnan(y[-2]) and torch.isnan(y[-1])
