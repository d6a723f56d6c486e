"""Conv1d kernels (NCL layout) over the native conv entry points.

Same classes and constructor signatures as the reference
(kernels/convolution/conv1d/conv1d.py:152-579):

* ``DepthwiseConv1dKernel`` (one channel per group) -> ``tileops_conv1d_depthwise_fwd``:
  the hot path, register/shared-memory halo, fused bias and optional SiLU,
  no padded workspace (the reference allocates ``xpad`` per call,
  conv1d.py:570-578).
* ``Conv1dPointwiseKernel``, ``Conv1dKernel``, ``Conv1dUnitStrideKernel``,
  ``GroupConv1dKernel`` -> ``tileops_conv1d_direct_fwd``: a direct fp32
  accumulation kernel on CUDA cores (correct for every geometry; these dense
  paths are not the depthwise hot path and are not tuned).

Output length: ``(l_in + pad_left + pad_right - dilation * (k - 1) - 1) // stride + 1``.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch

from tileops import _native
from tileops.kernels.kernel_base import Kernel, check_dtype

__all__ = [
    "Conv1dKernel",
    "Conv1dPointwiseKernel",
    "Conv1dUnitStrideKernel",
    "DepthwiseConv1dKernel",
    "GroupConv1dKernel",
]

_DTYPES = (torch.float16, torch.bfloat16)
_ACTIVATIONS = {None: 0, "silu": 1}


def _out_len(l_in: int, k: int, stride: int, pad_l: int, pad_r: int, dilation: int) -> int:
    return (l_in + pad_l + pad_r - dilation * (k - 1) - 1) // stride + 1


class _DirectConv1d(Kernel):
    """Grouped direct convolution (groups = 1 for the dense kernels)."""

    groups = 1

    def _setup(self, n, c_in, l_in, c_out, kernel_l, stride_l, pad_l, dtype, dilation_l,
               has_bias, config):
        check_dtype(self, dtype, _DTYPES)
        self.n = n
        self.c_in = c_in
        self.l_in = l_in
        self.c_out = c_out
        self.kernel_l = kernel_l
        self.stride_l = stride_l
        self.pad_l = tuple(pad_l)
        self.pad_left, self.pad_right = self.pad_l
        self.dilation_l = dilation_l
        self.dtype = dtype
        self.has_bias = has_bias
        self.out_l = _out_len(l_in, kernel_l, stride_l, self.pad_left, self.pad_right, dilation_l)
        self.init_config(config)

    def forward(
        self, x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor] = None
    ) -> torch.Tensor:
        x = x.contiguous()
        weight = weight.contiguous()
        bias = bias.contiguous() if bias is not None else None
        y = torch.empty((self.n, self.c_out, max(self.out_l, 0)), dtype=self.dtype, device=x.device)
        if y.numel() == 0:
            return y
        _native.launch(
            "tileops_conv1d_direct_fwd",
            x.device,
            _native.ptr(x),
            _native.ptr(weight),
            _native.ptr(bias),
            _native.ptr(y),
            self.n,
            self.c_in,
            self.l_in,
            self.c_out,
            self.out_l,
            self.kernel_l,
            self.stride_l,
            self.pad_left,
            self.dilation_l,
            self.groups,
            _native.dtype_code(self.dtype),
        )
        return y


class Conv1dPointwiseKernel(_DirectConv1d):
    """Dense 1x1 Conv1d (kernel 1, stride 1, no padding)."""

    def __init__(self, n: int, c_in: int, l_in: int, c_out: int, dtype: torch.dtype,
                 has_bias: bool = False, config: Optional[dict] = None) -> None:
        super().__init__()
        self._setup(n, c_in, l_in, c_out, 1, 1, (0, 0), dtype, 1, has_bias, config)


class Conv1dKernel(_DirectConv1d):
    """Dense Conv1d, any stride / padding / dilation."""

    def __init__(self, n: int, c_in: int, l_in: int, c_out: int, kernel_l: int,
                 stride_l: int, pad_l: Tuple[int, int], dtype: torch.dtype,
                 dilation_l: int = 1, has_bias: bool = False,
                 config: Optional[dict] = None) -> None:
        super().__init__()
        self._setup(n, c_in, l_in, c_out, kernel_l, stride_l, pad_l, dtype, dilation_l,
                    has_bias, config)


class Conv1dUnitStrideKernel(Conv1dKernel):
    """Dense Conv1d with stride 1."""


class GroupConv1dKernel(_DirectConv1d):
    """Grouped Conv1d (``groups > 1``)."""

    def __init__(self, n: int, c_in: int, l_in: int, c_out: int, kernel_l: int,
                 stride_l: int, pad_l: Tuple[int, int], dtype: torch.dtype,
                 dilation_l: int = 1, has_bias: bool = False, groups: int = 1,
                 c_in_g: Optional[int] = None, c_out_g: Optional[int] = None,
                 config: Optional[dict] = None) -> None:
        super().__init__()
        self.groups = groups
        self.c_in_g = c_in_g if c_in_g is not None else c_in // max(groups, 1)
        self.c_out_g = c_out_g if c_out_g is not None else c_out // max(groups, 1)
        if self.groups <= 1:
            raise ValueError(f"{type(self).__name__} requires groups > 1")
        if c_in % groups or c_out % groups:
            raise ValueError(
                f"{type(self).__name__} requires c_in and c_out divisible by groups; "
                f"got c_in={c_in}, c_out={c_out}, groups={groups}"
            )
        self._setup(n, c_in, l_in, c_out, kernel_l, stride_l, pad_l, dtype, dilation_l,
                    has_bias, config)


class DepthwiseConv1dKernel(GroupConv1dKernel):
    """Depthwise Conv1d: one input and one output channel per group.

    Extra keyword beyond the reference signature: ``activation`` (None or
    ``"silu"``), fused into the epilogue; used by the causal (Mamba-style)
    depthwise op.  Weights / bias may be the input dtype or float32.
    """

    SUPPORTED_ACTIVATIONS = tuple(_ACTIVATIONS)

    def __init__(self, n: int, c_in: int, l_in: int, c_out: int, kernel_l: int,
                 stride_l: int, pad_l: Tuple[int, int], dtype: torch.dtype,
                 dilation_l: int = 1, has_bias: bool = False, groups: int = 1,
                 c_in_g: Optional[int] = None, c_out_g: Optional[int] = None,
                 config: Optional[dict] = None, activation: Optional[str] = None) -> None:
        if activation not in _ACTIVATIONS:
            raise ValueError(f"unsupported activation {activation!r}; expected None or 'silu'")
        self.activation = activation
        super().__init__(n, c_in, l_in, c_out, kernel_l, stride_l, pad_l, dtype,
                         dilation_l=dilation_l, has_bias=has_bias, groups=groups,
                         c_in_g=c_in_g, c_out_g=c_out_g, config=config)
        if c_in != c_out or self.c_in_g != 1:
            raise ValueError(f"{type(self).__name__} requires c_in == c_out == groups")

    def forward(
        self, x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor] = None
    ) -> torch.Tensor:
        x = x.contiguous()
        weight = weight.contiguous()
        bias = bias.contiguous() if bias is not None else None
        if bias is not None and bias.dtype != weight.dtype:
            raise ValueError(f"bias.dtype {bias.dtype} must match weight.dtype {weight.dtype}")
        y = torch.empty((self.n, self.c_out, max(self.out_l, 0)), dtype=self.dtype, device=x.device)
        if y.numel() == 0:
            return y
        _native.launch(
            "tileops_conv1d_depthwise_fwd",
            x.device,
            _native.ptr(x),
            _native.ptr(weight),
            _native.ptr(bias),
            _native.ptr(y),
            self.n,
            self.c_in,
            self.l_in,
            self.out_l,
            self.kernel_l,
            self.stride_l,
            self.pad_left,
            self.dilation_l,
            _native.dtype_code(self.dtype),
            _native.dtype_code(weight.dtype),
            _ACTIVATIONS[self.activation],
        )
        return y
