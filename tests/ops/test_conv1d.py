"""GPU parity of Conv1dFwdOp / Conv1dBiasFwdOp and the causal depthwise op.

Ported from TO/tests/ops/test_conv1d.py (the Conv1dFixture sweep from
TO/tileops/workloads/convolution.py:20-242 and the explicit smoke tests:
no-bias / bias, dilation, 'same' with an even kernel, dispatch keys,
depthwise, grouped, dtype rejection, roofline), tolerances from
conv1d_tolerance, ref_program = oracle.  Added: reference-output fixtures,
the causal (Mamba-style) depthwise form with and without SiLU at small sizes
and at BASELINE's (8, 4096, 8192) size (every channel of one batch row
checked against the oracle: depthwise channels are independent).
"""

import pytest
import torch

from oracle import reference as ref
from tests.golden.load import load, names
from tileops.ops.convolution import CausalDepthwiseConv1dFwdOp, Conv1dBiasFwdOp, Conv1dFwdOp
from tileops.testing.test_base import TestBase
from tileops.workloads.convolution import (
    CausalConv1dWorkload,
    Conv1dFixture,
    Conv1dWorkload,
    conv1d_tolerance,
)

pytestmark = pytest.mark.gpu


class Conv1dTest(Conv1dWorkload, TestBase):
    def ref_program(self, x, weight, bias):
        return ref.conv1d(x, weight, bias, self.stride, self.padding, self.dilation, self.groups)


@Conv1dFixture
def test_conv1d(n, c_in, l_in, c_out, kernel_size, stride, padding, dilation, groups, dtype,
                use_bias):
    test = Conv1dTest(n, c_in, l_in, c_out, kernel_size, stride, padding, dilation, groups,
                      dtype, use_bias)
    op = Conv1dFwdOp(stride=stride, padding=padding, dilation=dilation, groups=groups)
    tol = conv1d_tolerance(dtype, padding=padding, kernel_shape=(kernel_size,))
    test.check(op, *test.gen_inputs(), atol=tol["atol"], rtol=tol["rtol"])


def _check(out, x, w, b=None, **kw):
    expect = ref.conv1d(x, w, b, **kw)
    tol = conv1d_tolerance(out.dtype, padding=kw.get("padding", 0),
                           kernel_shape=(w.shape[-1],))
    torch.testing.assert_close(out.cpu(), expect, atol=tol["atol"], rtol=tol["rtol"])


def test_conv1d_no_bias_and_bias():
    x = torch.randn(1, 32, 256, device="cuda", dtype=torch.float16)
    w = torch.randn(64, 32, 5, device="cuda", dtype=torch.float16)
    b = torch.randn(64, device="cuda", dtype=torch.float16)
    _check(Conv1dFwdOp(stride=2, padding=2)(x, w), x, w, stride=2, padding=2)
    _check(Conv1dFwdOp(stride=2, padding=2)(x, w, b), x, w, b, stride=2, padding=2)
    _check(Conv1dBiasFwdOp(stride=2, padding=2)(x, w, b), x, w, b, stride=2, padding=2)


@pytest.mark.parametrize("use_bias", [False, True])
def test_conv1d_dilation(use_bias):
    x = torch.randn(1, 32, 128, device="cuda", dtype=torch.float16)
    w = torch.randn(64, 32, 3, device="cuda", dtype=torch.float16)
    b = torch.randn(64, device="cuda", dtype=torch.float16) if use_bias else None
    _check(Conv1dFwdOp(padding=2, dilation=2)(x, w, b), x, w, b, padding=2, dilation=2)


@pytest.mark.parametrize("use_bias", [False, True])
def test_conv1d_same_padding_even_kernel(use_bias):
    x = torch.randn(1, 16, 129, device="cuda", dtype=torch.float16)
    w = torch.randn(32, 16, 2, device="cuda", dtype=torch.float16)
    b = torch.randn(32, device="cuda", dtype=torch.float16) if use_bias else None
    _check(Conv1dFwdOp(padding="same")(x, w, b), x, w, b, padding="same")


@pytest.mark.parametrize("kernel_size, stride, padding", [(3, 1, 1), (3, 2, 1), (1, 1, 0)])
def test_conv1d_dispatched_kernels_match(kernel_size, stride, padding):
    x = torch.randn(1, 32, 256, device="cuda", dtype=torch.float16)
    w = torch.randn(64, 32, kernel_size, device="cuda", dtype=torch.float16)
    _check(Conv1dFwdOp(stride=stride, padding=padding)(x, w), x, w, stride=stride,
           padding=padding)


def test_conv1d_depthwise():
    op = Conv1dFwdOp(padding=1, groups=32)
    x = torch.randn(1, 32, 128, device="cuda", dtype=torch.float16)
    w = torch.randn(32, 1, 3, device="cuda", dtype=torch.float16)
    out = op(x, w)
    assert type(op.kernel).__name__ == "DepthwiseConv1dKernel"
    _check(out, x, w, padding=1, groups=32)


@pytest.mark.parametrize("use_bias", [False, True])
def test_conv1d_grouped(use_bias):
    x = torch.randn(1, 32, 128, device="cuda", dtype=torch.float16)
    w = torch.randn(64, 16, 3, device="cuda", dtype=torch.float16)
    b = torch.randn(64, device="cuda", dtype=torch.float16) if use_bias else None
    _check(Conv1dFwdOp(padding=1, groups=2)(x, w, b), x, w, b, padding=1, groups=2)


def test_conv1d_rejects_fp32():
    x = torch.randn(1, 8, 32, device="cuda")
    with pytest.raises(ValueError, match="does not support dtype"):
        Conv1dFwdOp()(x, torch.randn(16, 8, 3, device="cuda"))


def test_conv1d_eval_roofline():
    n, c_in, l_in, c_out, k = 1, 32, 128, 64, 3
    op = Conv1dFwdOp(padding=0)
    op(torch.randn(n, c_in, l_in, device="cuda", dtype=torch.float16),
       torch.randn(c_out, c_in, k, device="cuda", dtype=torch.float16))
    out_l = l_in - k + 1
    flops, nbytes = op.eval_roofline()
    assert flops == 2 * n * c_out * c_in * out_l * k
    assert nbytes == (n * c_in * l_in + c_out * c_in * k + n * c_out * out_l) * 2


@pytest.mark.parametrize("name", [n for n in names("conv1d_") if "golden" not in n])
def test_reference_fixture(name):
    case = load(name)
    m, i = case["meta"], case["inputs"]
    x, w = i["x"].cuda(), i["weight"].cuda()
    b = i["bias"].cuda() if i["bias"] is not None else None
    op = Conv1dFwdOp(stride=m["stride"], padding=m["padding"], dilation=m["dilation"],
                     groups=m["groups"])
    y = op(x, w, b).cpu()
    tol = conv1d_tolerance(x.dtype, padding=m["padding"], kernel_shape=(m["kernel_size"],))
    torch.testing.assert_close(y, case["outputs"]["y"], atol=tol["atol"], rtol=tol["rtol"])


# ------------------------------------------------------ causal depthwise
def test_causal_matches_reference_depthwise_golden():
    case = load("conv1d_depthwise_golden_causal_bf16")
    i = case["inputs"]
    x = i["x"].cuda()
    y = CausalDepthwiseConv1dFwdOp()(x, i["weight"].cuda(), i["bias"].cuda())
    expect = case["outputs"]["y_full"][..., : x.shape[-1]]
    torch.testing.assert_close(y.cpu(), expect, atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("activation", [None, "silu"])
@pytest.mark.parametrize("width", [2, 3, 4, 5, 7, 9, 31])
@pytest.mark.parametrize("dtype,w_dtype", [(torch.bfloat16, torch.bfloat16),
                                           (torch.bfloat16, torch.float32),
                                           (torch.float16, torch.float16)])
@pytest.mark.parametrize("seq_len", [1, 8, 100, 2048])
def test_causal_depthwise(activation, width, dtype, w_dtype, seq_len):
    x, w, b = CausalConv1dWorkload(2, 48, seq_len, width, dtype, w_dtype).gen_inputs()
    y = CausalDepthwiseConv1dFwdOp(activation=activation)(x, w, b)
    expect = ref.causal_depthwise_conv1d(x, w, b, activation)
    assert y.shape == x.shape
    tol = conv1d_tolerance(dtype)
    torch.testing.assert_close(y.cpu(), expect, atol=tol["atol"], rtol=tol["rtol"])


def test_causal_no_bias_and_3d_weight():
    x, w, _ = CausalConv1dWorkload(1, 16, 64, 4, torch.bfloat16).gen_inputs()
    y = CausalDepthwiseConv1dFwdOp()(x, w.reshape(16, 1, 4))
    torch.testing.assert_close(y.cpu(), ref.causal_depthwise_conv1d(x, w), atol=2e-2, rtol=2e-2)


@pytest.mark.full
@pytest.mark.parametrize("activation", [None, "silu"])
def test_causal_baseline_config(activation):
    """BASELINE: x (8, 4096, 8192) bf16, w (4096, 4) ~ N(0, 0.25), b ~ N(0, 0.01)."""
    x, w, b = CausalConv1dWorkload(8, 4096, 8192, 4, torch.bfloat16).gen_inputs()
    op = CausalDepthwiseConv1dFwdOp(activation=activation)
    y = op(x, w, b)
    for row in (0, 7):  # every channel of two batch rows
        expect = ref.causal_depthwise_conv1d(x[row : row + 1], w, b, activation)
        torch.testing.assert_close(y[row : row + 1].cpu(), expect, atol=2e-2, rtol=2e-2)
    flops, nbytes = op.eval_roofline()
    assert nbytes == 2 * x.numel() * 2 + 4096 * 5 * 2
