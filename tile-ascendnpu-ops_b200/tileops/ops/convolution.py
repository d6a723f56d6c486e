"""Convolution operators (NCL layout).

``Conv1dFwdOp`` / ``Conv1dBiasFwdOp`` keep the reference API
(ops/convolution.py:74-383): ``Conv1dFwdOp(stride=1, padding=0, dilation=1,
groups=1, kernel_map=None)`` with ``padding`` an int, a 1-tuple, ``'valid'``
or ``'same'`` (extra element of an odd total on the right), kernel selection
by ``_select_kernel_key`` (depthwise when every group has one input and one
output channel), a per-geometry kernel cache, and ``eval_roofline`` after a
forward (one multiply-add per in-range tap, each tensor moved once, the input
counted only at positions some window reads).

``CausalDepthwiseConv1dFwdOp`` is this build's explicit extension for the
causal (Mamba-style) depthwise convolution the reference API cannot express
(``padding`` there pads both sides): left padding ``k - 1``, no right
padding, output length ``l_in``, optional fused SiLU; weight ``(C, k)`` or
``(C, 1, k)`` in the input dtype or float32.  It runs the same
``depthwise_conv1d`` kernel.
"""

from __future__ import annotations

from typing import Dict, Optional, Tuple

import torch

from tileops.device import get_device_backend
from tileops.kernels.convolution import (
    Conv1dKernel,
    Conv1dPointwiseKernel,
    Conv1dUnitStrideKernel,
    DepthwiseConv1dKernel,
    GroupConv1dKernel,
)
from tileops.kernels.kernel_base import Kernel
from tileops.ops.op_base import Op

__all__ = ["CausalDepthwiseConv1dFwdOp", "Conv1dBiasFwdOp", "Conv1dFwdOp"]


def _axes(value, dims: int) -> Tuple[int, ...]:
    """A per-axis parameter as one value per spatial axis."""
    return (value,) * dims if isinstance(value, int) else tuple(value)


def _out_dim(size: int, kernel: int, stride: int, before: int, after: int, dilation: int) -> int:
    return (size + before + after - dilation * (kernel - 1) - 1) // stride + 1


def _tap_range(extent: int, out: int, j: int, stride: int, padding: int, dilation: int):
    """Outputs ``o`` in ``[lo, hi)`` whose tap ``j`` lands inside ``[0, extent)``."""
    off = j * dilation - padding  # input position of output 0's tap j
    lo = 0 if off >= 0 else (-off + stride - 1) // stride  # first o with o*stride + off >= 0
    last = extent - 1 - off  # o*stride must not exceed this
    hi = min(out, last // stride + 1) if last >= 0 else 0
    return lo, max(lo, hi), off


def _window_taps(extent: int, out: int, kernel: int, stride: int, padding: int, dilation: int) -> int:
    """In-range (output, tap) pairs over the axis; padded taps count none."""
    total = 0
    for j in range(kernel):
        lo, hi, _ = _tap_range(extent, out, j, stride, padding, dilation)
        total += hi - lo
    return total


def _window_reads(extent: int, out: int, kernel: int, stride: int, padding: int, dilation: int) -> int:
    """Distinct input positions the windows of the axis read."""
    hit = bytearray(extent)
    for j in range(kernel):
        lo, hi, off = _tap_range(extent, out, j, stride, padding, dilation)
        if hi > lo:
            start = lo * stride + off
            hit[start : (hi - 1) * stride + off + 1 : stride] = b"\x01" * (hi - lo)
    return sum(hit)


class Conv1dFwdOp(Op):
    """1-D convolution over an NCL input, as ``torch.nn.functional.conv1d``.

    Args:
        stride: Stride, an int or a 1-tuple (default 1).
        padding: Padding each side (int / 1-tuple), or ``'valid'`` / ``'same'``.
        dilation: Dilation, an int or a 1-tuple (default 1).
        groups: Number of channel groups (default 1).
        kernel_map: Optional override for kernel dispatch.
    """

    _SUPPORTED_DTYPES = (torch.float16, torch.bfloat16)

    def __init__(
        self,
        stride=1,
        padding=0,
        dilation=1,
        groups: int = 1,
        kernel_map: Optional[Dict[str, Kernel]] = None,
    ) -> None:
        self.stride = stride
        self.padding = padding
        self.dilation = dilation
        self.groups = groups
        self.dispatch_kernel(kernel_map)
        self._kernel_cache: Dict[tuple, Kernel] = {}
        self.kernel: Optional[Kernel] = None
        self.n = None
        self.c_in = None
        self.l_in = None
        self.c_out = None
        self.c_in_g = None
        self.c_out_g = None
        self.kernel_l = None
        self.stride_l = None
        self.dilation_l = None
        self.pad_left = None
        self.pad_right = None
        self.out_l = None
        self.has_bias = False
        self.dtype = None

    @property
    def default_kernel_map(self) -> Dict[str, Kernel]:
        return {
            "conv1d_pointwise": Conv1dPointwiseKernel,
            "conv1d": Conv1dKernel,
            "conv1d_unit_stride": Conv1dUnitStrideKernel,
            "depthwise_conv1d": DepthwiseConv1dKernel,
            "group_conv1d": GroupConv1dKernel,
        }

    def _select_kernel_key(self, c_in, c_in_g, c_out_g, kernel_l, stride, pad_left,
                           pad_right, dilation) -> str:
        """The most specific kernel for this call (reference order)."""
        if self.groups > 1:
            if c_in_g == 1 and c_out_g == 1:
                return "depthwise_conv1d"
            return "group_conv1d"
        if kernel_l == 1 and stride == 1 and pad_left == 0 and pad_right == 0 and dilation == 1:
            return "conv1d_pointwise"
        if stride == 1 and kernel_l > 1 and c_in >= 16:
            return "conv1d_unit_stride"
        return "conv1d"

    def _get_kernel(self, key, n, c_in, l_in, c_out, c_in_g, c_out_g, kernel_l, stride, pad_l,
                    dilation, dtype, has_bias) -> Kernel:
        cache_key = (key, n, c_in, l_in, c_out, c_in_g, c_out_g, kernel_l, stride, pad_l,
                     dilation, dtype, has_bias)
        if cache_key in self._kernel_cache:
            return self._kernel_cache[cache_key]
        cls = self.kernel_map[key]
        if key == "conv1d_pointwise":
            kernel = cls(n, c_in, l_in, c_out, dtype, has_bias=has_bias)
        elif key in ("conv1d", "conv1d_unit_stride"):
            kernel = cls(n, c_in, l_in, c_out, kernel_l, stride, pad_l, dtype,
                         dilation_l=dilation, has_bias=has_bias)
        else:
            kernel = cls(n, c_in, l_in, c_out, kernel_l, stride, pad_l, dtype,
                         dilation_l=dilation, has_bias=has_bias, groups=self.groups,
                         c_in_g=c_in_g, c_out_g=c_out_g)
        self._kernel_cache[cache_key] = kernel
        return kernel

    def _resolve_geometry(self, l_in: int, kernel_l: int) -> tuple[int, int, int, int, int]:
        (stride,) = _axes(self.stride, 1)
        (dilation,) = _axes(self.dilation, 1)
        if self.padding == "same":
            total = dilation * (kernel_l - 1)
            pad_left, pad_right, out_l = total // 2, total - total // 2, l_in
        else:
            (pad,) = (0,) if self.padding == "valid" else _axes(self.padding, 1)
            pad_left = pad_right = pad
            out_l = _out_dim(l_in, kernel_l, stride, pad, pad, dilation)
        return stride, dilation, pad_left, pad_right, out_l

    def forward(
        self,
        input: torch.Tensor,
        weight: torch.Tensor,
        bias: Optional[torch.Tensor] = None,
    ) -> torch.Tensor:
        """``input`` (N, C_in, L), ``weight`` (C_out, C_in/groups, k) -> (N, C_out, L_out)."""
        backend = get_device_backend()
        if not backend.is_device_tensor(input):
            raise ValueError(f"input must be a {backend.name} tensor, got device {input.device}")
        if input.dtype not in self._SUPPORTED_DTYPES:
            names = ", ".join(str(dt) for dt in self._SUPPORTED_DTYPES)
            raise ValueError(
                f"{type(self).__name__} does not support dtype {input.dtype}. "
                f"Supported: [{names}]"
            )
        if input.ndim != 3:
            raise ValueError("input must have shape [N, C_in, L_in]")
        n, c_in, l_in = input.shape
        c_out, c_in_g, kernel_l = weight.shape
        stride, dilation, pad_left, pad_right, out_l = self._resolve_geometry(l_in, kernel_l)
        c_out_g = c_out // self.groups
        key = self._select_kernel_key(c_in, c_in_g, c_out_g, kernel_l, stride, pad_left,
                                      pad_right, dilation)
        kernel = self._get_kernel(key, n, c_in, l_in, c_out, c_in_g, c_out_g, kernel_l, stride,
                                  (pad_left, pad_right), dilation, input.dtype,
                                  bias is not None)
        self.n, self.c_in, self.l_in, self.c_out = n, c_in, l_in, c_out
        self.c_in_g, self.c_out_g, self.kernel_l = c_in_g, c_out_g, kernel_l
        self.stride_l, self.dilation_l = stride, dilation
        self.pad_left, self.pad_right, self.out_l = pad_left, pad_right, out_l
        self.has_bias = bias is not None
        self.dtype = input.dtype
        self.kernel = kernel
        return kernel(input.contiguous(), weight.contiguous(),
                      bias.contiguous() if bias is not None else None)

    def eval_roofline(self) -> tuple[int, int]:
        """``(flops, bytes)`` of the last forwarded call."""
        if self.dtype is None:
            raise RuntimeError(
                f"{type(self).__name__}.eval_roofline() requires a prior forward() "
                "call to bind dynamic input shape"
            )
        n, c_in, l_in, c_out = int(self.n), int(self.c_in), int(self.l_in), int(self.c_out)
        c_in_g, kernel_l = int(self.c_in_g), int(self.kernel_l)
        stride, dilation, out_l = int(self.stride_l), int(self.dilation_l), int(self.out_l)
        eb = self.dtype.itemsize
        taps = _window_taps(l_in, out_l, kernel_l, stride, self.pad_left, dilation)
        flops = 2 * n * c_out * c_in_g * taps
        if self.has_bias:
            flops += n * c_out * out_l
        input_bytes = n * c_in * l_in * eb
        total_bytes = (
            n * c_in * l_in + c_out * c_in_g * kernel_l + n * c_out * out_l
            + (c_out if self.has_bias else 0)
        ) * eb
        reads = _window_reads(l_in, out_l, kernel_l, stride, self.pad_left, dilation)
        nbytes = total_bytes - input_bytes + input_bytes * reads // max(l_in, 1)
        return int(flops), int(nbytes)


class Conv1dBiasFwdOp(Conv1dFwdOp):
    """Conv1d with a required per-output-channel bias (reference ops/convolution.py:332-383)."""

    def forward(self, input: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
        if bias is None:
            raise ValueError("Conv1dBiasFwdOp requires a bias tensor; got None")
        backend = get_device_backend()
        if not backend.is_device_tensor(bias):
            raise ValueError(f"bias must be a {backend.name} tensor, got device {bias.device}")
        if bias.dtype != input.dtype:
            raise ValueError(f"bias.dtype {bias.dtype} must match input.dtype {input.dtype}")
        if bias.device != input.device:
            raise ValueError(f"bias.device {bias.device} must match input.device {input.device}")
        if weight.ndim < 1:
            raise ValueError("weight must have shape [C_out, C_in / groups, k]")
        c_out = weight.shape[0]
        if bias.ndim != 1 or bias.shape[0] != c_out:
            raise ValueError(f"bias must have shape [C_out] = [{c_out}], got {tuple(bias.shape)}")
        return super().forward(input, weight, bias)


class CausalDepthwiseConv1dFwdOp(Op):
    """Causal depthwise conv1d with optional fused SiLU (Mamba ``causal_conv1d``).

    ``out[b, c, l] = act(bias[c] + sum_k w[c, k] * x[b, c, l - (K-1) + k])``
    with ``x`` zero for negative positions; output shape equals ``x``'s.

    Args:
        activation: None or ``"silu"``.
        kernel_map: Optional override of ``"depthwise_conv1d"``.
    """

    _SUPPORTED_DTYPES = (torch.float16, torch.bfloat16)

    def __init__(self, activation: Optional[str] = None,
                 kernel_map: Optional[Dict[str, Kernel]] = None) -> None:
        if activation not in (None, "silu"):
            raise ValueError(f"unsupported activation {activation!r}; expected None or 'silu'")
        self.activation = activation
        self.dispatch_kernel(kernel_map)
        self._kernel_cache: Dict[tuple, Kernel] = {}
        self.kernel: Optional[Kernel] = None
        self.dtype = None
        self.shape = None
        self.kernel_l = None
        self.has_bias = False
        self.w_itemsize = None

    @property
    def default_kernel_map(self) -> Dict[str, Kernel]:
        return {"depthwise_conv1d": DepthwiseConv1dKernel}

    def forward(self, x: torch.Tensor, weight: torch.Tensor,
                bias: Optional[torch.Tensor] = None) -> torch.Tensor:
        backend = get_device_backend()
        for name, t in (("x", x), ("weight", weight), ("bias", bias)):
            if t is not None and not backend.is_device_tensor(t):
                raise ValueError(f"{name} must be a {backend.name} tensor, got device {t.device}")
        if x.dtype not in self._SUPPORTED_DTYPES:
            names = ", ".join(str(dt) for dt in self._SUPPORTED_DTYPES)
            raise ValueError(
                f"{type(self).__name__} does not support dtype {x.dtype}. Supported: [{names}]"
            )
        if x.ndim != 3:
            raise ValueError("x must have shape [B, C, L]")
        b, c, l_in = x.shape
        if weight.ndim == 3 and weight.shape[1] == 1:
            weight = weight.reshape(weight.shape[0], weight.shape[2])
        if weight.ndim != 2 or weight.shape[0] != c:
            raise ValueError(f"weight must have shape [C, k] = [{c}, k], got {tuple(weight.shape)}")
        if weight.dtype not in (x.dtype, torch.float32):
            raise ValueError(f"weight.dtype {weight.dtype} must be {x.dtype} or torch.float32")
        if bias is not None:
            if bias.shape != (c,):
                raise ValueError(f"bias must have shape [C] = [{c}], got {tuple(bias.shape)}")
            if bias.dtype != weight.dtype:
                raise ValueError(f"bias.dtype {bias.dtype} must match weight.dtype {weight.dtype}")
        k = weight.shape[1]
        key = (b, c, l_in, k, x.dtype, bias is not None)
        kernel = self._kernel_cache.get(key)
        if kernel is None:
            kernel = self.kernel_map["depthwise_conv1d"](
                b, c, l_in, c, k, 1, (k - 1, 0), x.dtype, dilation_l=1,
                has_bias=bias is not None, groups=c, c_in_g=1, c_out_g=1,
                activation=self.activation,
            )
            self._kernel_cache[key] = kernel
        self.kernel = kernel
        self.dtype, self.shape, self.kernel_l = x.dtype, (b, c, l_in), k
        self.has_bias, self.w_itemsize = bias is not None, weight.dtype.itemsize
        return kernel(x, weight, bias)

    def eval_roofline(self) -> tuple[int, int]:
        """Flops: 2 per in-range tap (+1 per output for the bias); bytes: x, y, w, b once."""
        if self.dtype is None:
            raise RuntimeError(
                f"{type(self).__name__}.eval_roofline() requires a prior forward() call"
            )
        b, c, l_in = self.shape
        k = self.kernel_l
        taps = _window_taps(l_in, l_in, k, 1, k - 1, 1)
        flops = 2 * b * c * taps + (b * c * l_in if self.has_bias else 0)
        eb = self.dtype.itemsize
        nbytes = 2 * b * c * l_in * eb + c * k * self.w_itemsize
        if self.has_bias:
            nbytes += c * self.w_itemsize
        return int(flops), int(nbytes)
