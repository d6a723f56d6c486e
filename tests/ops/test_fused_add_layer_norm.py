"""GPU parity of FusedAddLayerNormFwdOp.

Ported from TO/tests/ops/test_fused_add_layer_norm.py: the (m, n, dtype)
sweep incl. non-power-of-two N=5120 and tail M=1025, the 3-D input case, the
root (16, 1152) shape, the two-output kernel contract and the roofline after
forward; tolerances fp32 1e-5, fp16 1e-3, bf16 1.6e-2; ref_program = oracle.
Added: reference-output fixtures, fp32 affine parameters (BASELINE config,
checked in full at (8192, 4096)), ragged N (scalar path), rows wider than the
register path, and run-to-run determinism.
"""

import pytest
import torch

from oracle import reference as ref
from tests.golden.load import load, names
from tileops.kernels.norm import FusedAddLayerNormKernel
from tileops.ops.norm import FusedAddLayerNormFwdOp
from tileops.testing.test_base import TestBase
from tileops.workloads.norm import FusedAddLayerNormWorkload

pytestmark = pytest.mark.gpu

TOL = {torch.float32: (1e-5, 1e-5), torch.float16: (1e-3, 1e-3), torch.bfloat16: (1.6e-2, 1.6e-2)}


class FusedAddLayerNormTest(FusedAddLayerNormWorkload, TestBase):
    def ref_program(self, x, residual, weight, bias):
        return ref.fused_add_layer_norm(x, residual, weight, bias, self.eps)


PARAMS = [
    pytest.param(64, 4096, torch.float32, marks=pytest.mark.smoke),
    pytest.param(64, 4096, torch.float16, marks=pytest.mark.smoke),
    pytest.param(64, 4096, torch.bfloat16, marks=pytest.mark.smoke),
    pytest.param(2048, 4096, torch.float16, marks=pytest.mark.full),
    pytest.param(2048, 4096, torch.bfloat16, marks=pytest.mark.full),
    pytest.param(2048, 5120, torch.float32, marks=pytest.mark.full),
    pytest.param(1025, 4096, torch.float16, marks=pytest.mark.full),
    pytest.param(2048, 8192, torch.bfloat16, marks=pytest.mark.full),
    pytest.param(1, 8192, torch.bfloat16, marks=pytest.mark.full),
]


@pytest.mark.parametrize("m, n, dtype", PARAMS)
def test_fused_add_layer_norm_op(m, n, dtype):
    test = FusedAddLayerNormTest(m, n, dtype)
    atol, rtol = TOL[dtype]
    test.check(FusedAddLayerNormFwdOp(dtype=dtype), *test.gen_inputs(), atol=atol, rtol=rtol)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_fused_add_layer_norm_3d(dtype):
    b, s, h = 2, 512, 4096
    x = torch.randn(b, s, h, dtype=dtype, device="cuda")
    r = torch.randn(b, s, h, dtype=dtype, device="cuda")
    w = torch.randn(h, dtype=dtype, device="cuda")
    bias = torch.randn(h, dtype=dtype, device="cuda")
    y_ref, added_ref = ref.fused_add_layer_norm(x, r, w, bias)
    y, residual_out = FusedAddLayerNormFwdOp(dtype=dtype)(x, r, w, bias)
    atol, rtol = TOL[dtype]
    assert y.shape == x.shape and residual_out.shape == x.shape
    torch.testing.assert_close(y.cpu(), y_ref, atol=atol, rtol=rtol)
    torch.testing.assert_close(residual_out.cpu(), added_ref, atol=atol, rtol=rtol)


def test_root_shape():
    test = FusedAddLayerNormTest(16, 1152, torch.float16)
    test.check(FusedAddLayerNormFwdOp(dtype=torch.float16), *test.gen_inputs(), atol=1e-3,
               rtol=1e-3)


def test_eval_roofline_after_forward():
    m, n, dtype = 64, 4096, torch.float16
    op = FusedAddLayerNormFwdOp(dtype=dtype)
    op(*FusedAddLayerNormTest(m, n, dtype).gen_inputs())
    assert op.eval_roofline() == (8 * m * n, (4 * m * n + 2 * n) * 2)


def test_kernel_returns_two_outputs():
    m, n, dtype = 8, 4096, torch.float16
    test = FusedAddLayerNormTest(m, n, dtype)
    outputs = FusedAddLayerNormKernel(m, n, test.eps, dtype)(*test.gen_inputs())
    assert isinstance(outputs, list) and len(outputs) == 2
    assert all(out.shape == (m, n) for out in outputs)


@pytest.mark.parametrize("name", names("fused_add_layer_norm_"))
def test_reference_fixture(name):
    case = load(name)
    i = {k: v.cuda() for k, v in case["inputs"].items()}
    y, added = FusedAddLayerNormFwdOp(dtype=i["x"].dtype, eps=case["meta"]["eps"])(
        i["x"], i["residual"], i["weight"], i["bias"])
    atol, rtol = TOL[i["x"].dtype]
    torch.testing.assert_close(y.cpu(), case["outputs"]["y"], atol=atol, rtol=rtol)
    # The rounded sum is an exact op: bit-identical.
    assert torch.equal(added.cpu(), case["outputs"]["residual_out"])


@pytest.mark.parametrize("m, n", [(8192, 4096), (3, 4096)])
def test_fp32_affine_baseline_config(m, n):
    """BASELINE config: bf16 rows, fp32 weight = 1 + 0.1 N(0,1), bias = 0.1 N(0,1)."""
    x = torch.randn(m, n, dtype=torch.bfloat16, device="cuda")
    r = torch.randn(m, n, dtype=torch.bfloat16, device="cuda")
    w = 1.0 + 0.1 * torch.randn(n, device="cuda")
    b = 0.1 * torch.randn(n, device="cuda")
    op = FusedAddLayerNormFwdOp(dtype=torch.bfloat16)
    y, added = op(x, r, w, b)
    y_ref, added_ref = ref.fused_add_layer_norm(x, r, w, b)
    torch.testing.assert_close(y.cpu(), y_ref, atol=1.6e-2, rtol=1.6e-2)
    assert torch.equal(added.cpu(), added_ref)
    assert op.eval_roofline() == (8 * m * n, 4 * m * n * 2 + 2 * n * 4)


@pytest.mark.parametrize("n", [1, 5, 100, 1000, 4097])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_ragged_hidden(n, dtype):
    test = FusedAddLayerNormTest(7, n, dtype)
    atol, rtol = TOL[dtype]
    test.check(FusedAddLayerNormFwdOp(dtype=dtype), *test.gen_inputs(), atol=atol, rtol=rtol)


@pytest.mark.parametrize("n", [65_536 + 8, 100_000])
def test_wide_rows(n):
    test = FusedAddLayerNormTest(3, n, torch.bfloat16)
    test.check(FusedAddLayerNormFwdOp(dtype=torch.bfloat16), *test.gen_inputs(), atol=1.6e-2,
               rtol=1.6e-2)


def test_deterministic():
    inputs = FusedAddLayerNormTest(256, 4096, torch.bfloat16).gen_inputs()
    op = FusedAddLayerNormFwdOp(dtype=torch.bfloat16)
    outs = [op(*inputs) for _ in range(3)]
    for y, s in outs[1:]:
        assert torch.equal(y, outs[0][0]) and torch.equal(s, outs[0][1])


@pytest.mark.parametrize("n", [1024, 1032, 2000, 3000, 4096])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("f32_affine", [False, True])
def test_many_rows_per_width(n, dtype, f32_affine):
    """Enough rows for the persistent ring kernel at widths of 1024..4096,
    including widths whose last thread packets are partly empty; weight and
    bias in the row dtype or fp32; residual_out bit-exact, y at the
    reference tolerance."""
    m = 700
    x = torch.randn(m, n, dtype=dtype, device="cuda")
    r = torch.randn(m, n, dtype=dtype, device="cuda")
    wdt = torch.float32 if f32_affine else dtype
    w = (1.0 + 0.1 * torch.randn(n, device="cuda")).to(wdt)
    b = (0.1 * torch.randn(n, device="cuda")).to(wdt)
    y, added = FusedAddLayerNormFwdOp(dtype=dtype)(x, r, w, b)
    y_ref, added_ref = ref.fused_add_layer_norm(x, r, w, b)
    atol, rtol = TOL[dtype]
    torch.testing.assert_close(y.cpu(), y_ref, atol=atol, rtol=rtol)
    assert torch.equal(added.cpu(), added_ref)
