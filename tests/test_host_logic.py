"""Host-side contract of the ops, ported from the reference tests' API checks
(no kernel launches, CPU only): dtype rejection messages, constructor
contracts, roofline formulas, kernel dispatch keys and validation errors
raised before any launch."""

from math import prod

import pytest
import torch

from tileops.benchmark.msprof import _extract_op_init_args
from tileops.kernels.attention.multi_head_attention import GQAPrefillFwdKernel
from tileops.kernels.elementwise import (
    BitwiseNotFwdKernel,
    ClampScalarFwdKernel,
    GeluAndMulFwdKernel,
    GeluTanhAndMulFwdKernel,
    HardsigmoidFwdKernel,
    HardswishFwdKernel,
    IsfiniteFwdKernel,
    IsinfFwdKernel,
    IsnanFwdKernel,
)
from tileops.kernels.norm import FusedAddLayerNormKernel
from tileops.manifest import load_manifest, load_workloads
from tileops.ops.attention import MultiHeadAttentionFwdOp
from tileops.ops.convolution import CausalDepthwiseConv1dFwdOp, Conv1dBiasFwdOp, Conv1dFwdOp
from tileops.ops.elementwise import (
    BitwiseNotFwdOp,
    ClampMinFwdOp,
    ClampScalarFwdOp,
    GeluAndMulFwdOp,
    GeluTanhAndMulFwdOp,
    HardsigmoidFwdOp,
    HardswishFwdOp,
    IsfiniteFwdOp,
    IsinfFwdOp,
    IsnanFwdOp,
)
from tileops.ops.norm import FusedAddLayerNormFwdOp


# ------------------------------------------------------------ dtype gates
@pytest.mark.parametrize(
    "kernel_cls",
    [HardswishFwdKernel, HardsigmoidFwdKernel, IsnanFwdKernel, IsinfFwdKernel,
     IsfiniteFwdKernel],
)
def test_float_unary_kernels_reject_int(kernel_cls):
    with pytest.raises(ValueError, match="only supports dtypes"):
        kernel_cls(N_total=16, dtype=torch.int32)


def test_clamp_kernel_rejects_int_and_missing_bounds():
    with pytest.raises(ValueError, match="only supports dtypes"):
        ClampScalarFwdKernel(N_total=16, dtype=torch.int32, min_val=-0.5)
    with pytest.raises(ValueError, match=r"present\(min\) or present\(max\)"):
        ClampScalarFwdOp(N_total=16, dtype=torch.float32, min=None, max=None)


def test_clamp_min_requires_min():
    with pytest.raises(ValueError, match="requires min"):
        ClampMinFwdOp(N_total=16, dtype=torch.float32)


def test_bitwise_not_rejects_float():
    with pytest.raises(ValueError, match="only supports dtypes"):
        BitwiseNotFwdKernel(N_total=16, dtype=torch.float32)
    with pytest.raises(ValueError, match="does not support dtype"):
        BitwiseNotFwdOp(N_total=16, dtype=torch.float32)


@pytest.mark.parametrize("op_cls", [IsnanFwdOp, IsinfFwdOp, IsfiniteFwdOp])
def test_predicate_ops_reject_int(op_cls):
    with pytest.raises(ValueError, match="does not support dtype"):
        op_cls(N_total=16, dtype=torch.int32)


@pytest.mark.parametrize(
    "op_cls,kernel_cls",
    [(GeluAndMulFwdOp, GeluAndMulFwdKernel), (GeluTanhAndMulFwdOp, GeluTanhAndMulFwdKernel)],
)
def test_gated_reject_int(op_cls, kernel_cls):
    with pytest.raises(ValueError, match="does not support dtype"):
        op_cls(M=16, N=16, dtype=torch.int32)
    with pytest.raises(ValueError, match="only supports dtypes"):
        kernel_cls(M=16, N=16, dtype=torch.int32)


def test_norm_and_attention_kernels_reject_int():
    with pytest.raises(ValueError, match="only supports dtypes"):
        FusedAddLayerNormKernel(4, 8, 1e-5, torch.int32)
    with pytest.raises(ValueError, match="only supports dtypes"):
        GQAPrefillFwdKernel(1, 2, 2, 8, 8, 64, False, torch.float32)


# ------------------------------------------------------- roofline formulas
@pytest.mark.parametrize(
    "op_cls,fpe", [(HardswishFwdOp, 4), (HardsigmoidFwdOp, 3)]
)
def test_activation_roofline(op_cls, fpe):
    n = 1_048_576
    op = op_cls(N_total=n, dtype=torch.float16)
    assert op.eval_roofline() == (fpe * n, 2 * n * 2)


def test_clamp_roofline():
    n = 1_048_576
    op = ClampScalarFwdOp(N_total=n, dtype=torch.float16, min=-0.5, max=0.5)
    assert op.eval_roofline() == (n, 2 * n * 2)


@pytest.mark.parametrize("op_cls", [IsnanFwdOp, IsinfFwdOp, IsfiniteFwdOp])
def test_predicate_roofline(op_cls):
    n = 1_048_576
    op = op_cls(N_total=n, dtype=torch.float16)
    assert op.eval_roofline() == (n, n * (2 + 1))


def test_bitwise_not_roofline():
    n = 1_048_576
    op = BitwiseNotFwdOp(N_total=n, dtype=torch.int32)
    assert op.eval_roofline() == (n, 2 * n * 4)


@pytest.mark.parametrize("op_cls,fpo", [(GeluAndMulFwdOp, 6), (GeluTanhAndMulFwdOp, 10)])
def test_gated_roofline_and_init_args(op_cls, fpo):
    m, n, dtype = 64, 128, torch.float16
    op = op_cls(M=m, N=n, dtype=dtype)
    assert op.eval_roofline() == (fpo * m * n, 3 * m * n * 2)
    assert op.N_total == m * n and prod(op.out_shape) == m * n
    assert _extract_op_init_args(op) == {"M": m, "N": n, "dtype": dtype}


def test_faln_roofline_requires_forward():
    op = FusedAddLayerNormFwdOp(dtype=torch.float16)
    with pytest.raises(RuntimeError, match="requires a prior"):
        op.eval_roofline()


def test_mha_roofline_and_dispatch():
    batch, seq_len, heads, dim = 2, 512, 8, 64
    for is_causal in (True, False):
        op = MultiHeadAttentionFwdOp(batch, heads, seq_len, dim, is_causal, torch.float16)
        full = 4 * batch * heads * seq_len * seq_len * dim
        q_elems = batch * seq_len * heads * dim
        assert op.eval_roofline() == (full // 2 if is_causal else full, 2 * (2 * q_elems) * 2)
    assert op.kernel.__class__.__name__.startswith("GQA")


def test_conv_roofline_requires_forward():
    with pytest.raises(RuntimeError, match="requires a prior"):
        Conv1dFwdOp().eval_roofline()


# ------------------------------------------------------ conv dispatch keys
@pytest.mark.parametrize(
    "kernel_size, stride, padding, dilation, expected_key",
    [(3, 1, 1, 1, "conv1d_unit_stride"), (3, 2, 1, 1, "conv1d"), (1, 1, 0, 1, "conv1d_pointwise")],
)
def test_conv1d_dispatch_key(kernel_size, stride, padding, dilation, expected_key):
    op = Conv1dFwdOp(stride=stride, padding=padding, dilation=dilation)
    key = op._select_kernel_key(32, 32, 64, kernel_size, stride, padding, padding, dilation)
    assert key == expected_key


def test_conv1d_depthwise_and_group_keys():
    assert Conv1dFwdOp(padding=1, groups=32)._select_kernel_key(32, 1, 1, 3, 1, 1, 1, 1) == (
        "depthwise_conv1d")
    assert Conv1dFwdOp(padding=1, groups=2)._select_kernel_key(32, 16, 32, 3, 1, 1, 1, 1) == (
        "group_conv1d")


# ----------------------------------------- validation before any launch
def test_forward_rejects_cpu_tensors():
    x = torch.randn(16)
    with pytest.raises(ValueError, match="must be a cuda tensor"):
        HardswishFwdOp(N_total=16, dtype=torch.float32)(x)
    with pytest.raises(ValueError, match="must be a cuda tensor"):
        GeluAndMulFwdOp(M=4, N=2, dtype=torch.float32)(torch.randn(4, 4))
    with pytest.raises(ValueError, match="must be a cuda tensor"):
        FusedAddLayerNormFwdOp(dtype=torch.float32)(x, x, x, x)
    with pytest.raises(ValueError, match="must be a cuda tensor"):
        Conv1dFwdOp()(torch.randn(1, 4, 8, dtype=torch.float16),
                      torch.randn(4, 4, 3, dtype=torch.float16))
    with pytest.raises(ValueError, match="must be a cuda tensor"):
        MultiHeadAttentionFwdOp(1, 2, 8, 64, False, torch.float16)(
            *(torch.randn(1, 8, 2, 64, dtype=torch.float16),) * 3)


class _AcceptCpu:
    """Backend stand-in whose device check admits CPU tensors, so the later
    dtype / shape checks can be exercised on a host without a GPU.  Every
    case below raises before the kernel is called."""

    name = "cuda"

    def is_device_tensor(self, t):
        return isinstance(t, torch.Tensor)

    def is_available(self):
        return False


@pytest.fixture
def accept_cpu(monkeypatch):
    import tileops.ops.convolution as conv_mod
    import tileops.ops.elementwise._gated as gated_mod
    import tileops.ops.elementwise._unary as unary_mod
    import tileops.ops.norm.fused_add_layer_norm as faln_mod

    fake = _AcceptCpu()
    for mod in (unary_mod, gated_mod, faln_mod, conv_mod):
        monkeypatch.setattr(mod, "get_device_backend", lambda: fake)


def test_gated_rejects_dtype_and_shape_mismatch(accept_cpu):
    op = GeluAndMulFwdOp(M=4, N=8, dtype=torch.float32)
    with pytest.raises(ValueError, match="x.dtype"):
        op(torch.randn(4, 16, dtype=torch.float16))
    with pytest.raises(ValueError, match="x.shape"):
        op(torch.randn(4, 18))


def test_unary_rejects_dtype_and_numel(accept_cpu):
    op = HardswishFwdOp(N_total=16, dtype=torch.float32)
    with pytest.raises(ValueError, match="input.dtype"):
        op(torch.randn(16, dtype=torch.float16))
    with pytest.raises(ValueError, match="Expected 16 elements"):
        op(torch.randn(17))


def test_faln_rejects_bad_inputs(accept_cpu):
    op = FusedAddLayerNormFwdOp(dtype=torch.float16)
    x = torch.randn(16, 64, dtype=torch.float16)
    w = torch.randn(64, dtype=torch.float16)
    with pytest.raises(ValueError, match="residual shape"):
        op(x, x[:, :32], w, w)
    with pytest.raises(ValueError, match="x.dtype"):
        op(x.float(), x.float(), w.float(), w.float())
    with pytest.raises(ValueError, match="weight.dtype"):
        op(x, x, w.bfloat16(), w.bfloat16())
    with pytest.raises(ValueError, match="weight shape"):
        op(x, x, w[:32], w)
    with pytest.raises(ValueError, match="Expected M=3"):
        FusedAddLayerNormFwdOp(M=3, dtype=torch.float16)(x, x, w, w)


def test_conv_rejects_bad_inputs(accept_cpu):
    x = torch.randn(1, 8, 32)
    with pytest.raises(ValueError, match="does not support dtype"):
        Conv1dFwdOp()(x, torch.randn(16, 8, 3))
    with pytest.raises(ValueError, match="requires a bias tensor"):
        Conv1dBiasFwdOp()(x.half(), torch.randn(16, 8, 3).half(), None)
    with pytest.raises(ValueError, match="bias must have shape"):
        Conv1dBiasFwdOp()(x.half(), torch.randn(16, 8, 3).half(), torch.randn(4).half())
    causal = CausalDepthwiseConv1dFwdOp(activation="silu")
    with pytest.raises(ValueError, match="weight must have shape"):
        causal(x.half(), torch.randn(4, 4).half())
    with pytest.raises(ValueError, match="unsupported activation"):
        CausalDepthwiseConv1dFwdOp(activation="gelu")


def test_mha_kernel_contract():
    with pytest.raises(ValueError, match="divisible"):
        GQAPrefillFwdKernel(1, 6, 4, 8, 8, 64, False, torch.float16)
    with pytest.raises(ValueError, match="seq_len_q <= seq_len_kv"):
        GQAPrefillFwdKernel(1, 4, 4, 16, 8, 64, True, torch.float16)


def test_manifest_covers_hot_path():
    ops = load_manifest()
    for name in ["HardswishFwdOp", "GeluAndMulFwdOp", "FusedAddLayerNormFwdOp",
                 "MultiHeadAttentionFwdOp", "CausalDepthwiseConv1dFwdOp",
                 "GatedDeltaNetPrefillFwdOp"]:
        assert name in ops and load_workloads(name)
