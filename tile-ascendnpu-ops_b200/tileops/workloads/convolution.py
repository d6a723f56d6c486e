"""Workloads of the convolution family (reference workloads/convolution.py).

``Conv1dFixture`` carries the reference's conv1d parameter sweep
(workloads/convolution.py:20-242): dense k3 TCN blocks, padding wider than
the row, pointwise, strided, dilated, valid / same padding, grouped and the
k31 conformer depthwise case.  ``CausalConv1dWorkload`` is the causal
depthwise (Mamba-style) input set: x ~ N(0, 1), weight ~ N(0, 0.25),
bias ~ N(0, 0.01).
"""

from typing import Optional

import torch

from tileops.device import get_device_backend
from tileops.workloads.workload_base import FixtureBase, WorkloadBase


def _p(*vals, marks=(), id=None):
    import pytest

    return pytest.param(*vals, marks=list(marks), id=id)


class Conv1dFixture(FixtureBase):
    @classmethod
    def get_params(cls):
        import pytest

        smoke, full = pytest.mark.smoke, pytest.mark.full
        f16, bf16 = torch.float16, torch.bfloat16
        names = ("n, c_in, l_in, c_out, kernel_size, stride, padding, dilation, groups, dtype, "
                 "use_bias")
        return [
            (
                names,
                [
                    _p(2, 64, 512, 128, 3, 1, 1, 1, 1, f16, False, marks=[smoke],
                       id="smoke-tcn-k3-s1-fp16"),
                    _p(2, 64, 512, 128, 3, 1, 1, 1, 1, bf16, False, marks=[smoke],
                       id="smoke-tcn-k3-s1-bf16"),
                    _p(1, 17, 5, 7, 3, 1, 5, 2, 1, f16, False, marks=[smoke],
                       id="smoke-padding-wider-than-row-fp16"),
                    _p(4, 256, 32000, 512, 1, 1, 0, 1, 1, f16, False, marks=[full],
                       id="full-convtasnet-pointwise-k1-s1-fp16"),
                    _p(4, 128, 4096, 256, 3, 1, 1, 1, 1, f16, False, marks=[full],
                       id="full-seanet-residual-k3-s1-fp16"),
                    _p(4, 64, 16000, 128, 5, 2, 2, 1, 1, f16, False, marks=[full],
                       id="full-audio-downsample-k5-s2-fp16"),
                    _p(1, 32, 256, 64, 7, 1, 3, 1, 1, f16, False, marks=[full],
                       id="full-small-seanet-stem-k7-s1-fp16"),
                    _p(2, 128, 4096, 256, 3, 2, 1, 1, 1, bf16, False, marks=[full],
                       id="full-sequence-downsample-k3-s2-bf16"),
                    _p(1, 32, 512, 64, 3, 1, 2, 2, 1, f16, False, marks=[full],
                       id="full-dilation-k3-d2-fp16"),
                    _p(1, 32, 128, 64, 3, 1, "valid", 1, 1, f16, False, marks=[full],
                       id="full-padding-valid-fp16"),
                    _p(1, 32, 128, 64, 3, 1, "same", 1, 1, f16, False, marks=[full],
                       id="full-padding-same-fp16"),
                    _p(1, 32, 128, 64, 3, 1, 1, 1, 2, f16, False, marks=[full],
                       id="full-groups2-k3-fp16"),
                    _p(1, 48, 128, 72, 3, 1, 1, 1, 3, f16, False, marks=[full],
                       id="full-groups3-coutg24-fp16"),
                    _p(1, 64, 128, 64, 31, 1, 15, 1, 64, f16, True, marks=[full],
                       id="full-conformer-depthwise-k31-fp16"),
                ],
            ),
        ]


class Conv1dWorkload(WorkloadBase):
    """NCL input, OIL weight, optional zero bias (reference convolution.py:245-291)."""

    def __init__(self, n, c_in, l_in, c_out, kernel_size, stride, padding, dilation, groups,
                 dtype, use_bias=False) -> None:
        self.n = n
        self.c_in = c_in
        self.l_in = l_in
        self.c_out = c_out
        self.kernel_size = kernel_size
        self.stride = stride
        self.padding = padding
        self.dilation = dilation
        self.groups = groups
        self.dtype = dtype
        self.use_bias = use_bias

    def gen_inputs(self) -> tuple[torch.Tensor, torch.Tensor, Optional[torch.Tensor]]:
        device = get_device_backend().name
        x = torch.randn(self.n, self.c_in, self.l_in, device=device, dtype=self.dtype)
        weight = torch.randn(self.c_out, self.c_in // self.groups, self.kernel_size,
                             device=device, dtype=self.dtype)
        bias = (torch.zeros(self.c_out, device=device, dtype=self.dtype)
                if self.use_bias else None)
        return x, weight, bias


class CausalConv1dWorkload(WorkloadBase):
    """Causal depthwise conv inputs: x (B, D, L), weight (D, K), bias (D,)."""

    def __init__(self, batch: int, dim: int, seq_len: int, width: int, dtype: torch.dtype,
                 w_dtype: Optional[torch.dtype] = None, use_bias: bool = True):
        self.batch = batch
        self.dim = dim
        self.seq_len = seq_len
        self.width = width
        self.dtype = dtype
        self.w_dtype = w_dtype or dtype
        self.use_bias = use_bias

    def gen_inputs(self):
        device = get_device_backend().name
        x = torch.randn(self.batch, self.dim, self.seq_len, device=device, dtype=self.dtype)
        w = (0.5 * torch.randn(self.dim, self.width, device=device)).to(self.w_dtype)
        b = ((0.1 * torch.randn(self.dim, device=device)).to(self.w_dtype)
             if self.use_bias else None)
        return x, w, b


def conv1d_tolerance(dtype: torch.dtype, *, padding=0, kernel_shape: tuple = ()) -> dict:
    """Tolerance against the fp32 reference (reference convolution.py:404-427)."""
    if dtype == torch.float16:
        if padding == "same" and any(k % 2 == 0 for k in kernel_shape):
            return {"atol": 2e-3, "rtol": 3e-3}
        return {"atol": 1e-2, "rtol": 1e-2}
    if dtype == torch.bfloat16:
        return {"atol": 2e-2, "rtol": 2e-2}
    return {"atol": 1e-4, "rtol": 1e-4}
