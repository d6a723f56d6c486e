"""FusedAddLayerNormFwdOp -- fused residual add + LayerNorm, two outputs.

Same API as the reference op (ops/norm/fused_add_layer_norm.py:39-189):
``FusedAddLayerNormFwdOp(M=None, N=None, dtype=None, eps=1e-5,
kernel_map=None)``, ``forward(x, residual, weight, bias) -> (y,
residual_out)`` with arbitrary leading dims, kernels cached per
``(M, N, dtype, device_index)``, and ``eval_roofline`` available after a
forward.

One documented superset of the reference contract: ``weight`` and ``bias``
may also be float32 when ``x`` is float16 / bfloat16 (fp32 LayerNorm affine
parameters, as in BASELINE's FusedAddLayerNorm config).  Any other dtype
mismatch raises the reference's ``"Expected weight.dtype ..."`` error.
"""

from typing import Dict, Optional

import torch

from tileops.device import get_device_backend
from tileops.kernels.kernel_base import Kernel
from tileops.kernels.norm import FusedAddLayerNormKernel

from ..op_base import Op

__all__ = ["FusedAddLayerNormFwdOp"]


class FusedAddLayerNormFwdOp(Op):
    """Fused residual addition and Layer Normalization.

    Args:
        M: Optional committed row count (product of the leading dims).
        N: Optional committed hidden dimension.
        dtype: float32, float16 or bfloat16 (inferred from ``x`` when None).
        eps: Epsilon for numerical stability.
        kernel_map: Optional kernel override dictionary.
    """

    _op_name = "fused_add_layer_norm"

    def __init__(
        self,
        M: Optional[int] = None,
        N: Optional[int] = None,
        dtype: Optional[torch.dtype] = None,
        eps: float = 1e-5,
        kernel_map: Optional[Dict[str, Kernel]] = None,
    ):
        self.M = M
        self.N = N
        self.dtype = dtype
        self._committed_M = M
        self._committed_N = N
        self._committed_dtype = dtype
        self.eps = eps
        self.dispatch_kernel(kernel_map)
        self._kernel_cache: Dict[tuple, Kernel] = {}
        self._last_roofline_mn: Optional[tuple[int, int]] = None
        self._affine_itemsize: Optional[int] = None

    @property
    def default_kernel_map(self) -> Dict[str, Kernel]:
        return {self._op_name: FusedAddLayerNormKernel}

    def eval_roofline(self) -> tuple[int, int]:
        """``(8 * M * N, (4 * M * N + 2 * N) * elem_bytes)`` for the last forward.

        With float32 affine parameters the ``2 * N`` term is counted at 4 bytes.
        """
        if self._last_roofline_mn is None or self.dtype is None:
            raise RuntimeError(
                f"{type(self).__name__}.eval_roofline() requires a prior "
                "forward() call to bind input shape and dtype"
            )
        M, N = self._last_roofline_mn
        eb = self.dtype.itemsize
        ab = self._affine_itemsize or eb
        return 8 * M * N, 4 * M * N * eb + 2 * N * ab

    def _get_kernel(self, M: int, N: int, dtype: torch.dtype, device_index) -> Kernel:
        key = (M, N, dtype, device_index)
        if key not in self._kernel_cache:
            self._kernel_cache[key] = self.kernel_map[self._op_name](M, N, self.eps, dtype)
        return self._kernel_cache[key]

    def forward(
        self,
        x: torch.Tensor,
        residual: torch.Tensor,
        weight: torch.Tensor,
        bias: torch.Tensor,
    ) -> tuple[torch.Tensor, torch.Tensor]:
        """Return ``(y, residual_out)``, both shaped like ``x``."""
        backend = get_device_backend()
        for name, t in (("x", x), ("residual", residual), ("weight", weight), ("bias", bias)):
            if not backend.is_device_tensor(t):
                raise ValueError(f"{name} must be a {backend.name} tensor")

        expected_dtype = self._committed_dtype
        if expected_dtype is not None and x.dtype != expected_dtype:
            raise ValueError(f"Expected x.dtype {expected_dtype}, got {x.dtype}")
        if expected_dtype is None:
            expected_dtype = x.dtype
        if residual.dtype != expected_dtype:
            raise ValueError(f"Expected residual.dtype {expected_dtype}, got {residual.dtype}")
        fp32_affine = (
            weight.dtype == torch.float32
            and bias.dtype == torch.float32
            and expected_dtype != torch.float32
        )
        if not fp32_affine:
            for name, t in (("weight", weight), ("bias", bias)):
                if t.dtype != expected_dtype:
                    raise ValueError(f"Expected {name}.dtype {expected_dtype}, got {t.dtype}")

        if residual.shape != x.shape:
            raise ValueError(f"Expected residual shape {x.shape}, got {residual.shape}")
        N = x.shape[-1]
        if tuple(weight.shape) != (N,):
            raise ValueError(f"Expected weight shape {(N,)}, got {tuple(weight.shape)}")
        if tuple(bias.shape) != (N,):
            raise ValueError(f"Expected bias shape {(N,)}, got {tuple(bias.shape)}")
        if self._committed_N is not None and self._committed_N != N:
            raise ValueError(f"Expected hidden dim {self._committed_N}, got {N}")

        orig_shape = x.shape
        x = x.contiguous().reshape(-1, N)
        residual = residual.contiguous().reshape(-1, N)
        M_actual = x.shape[0]
        if self._committed_M is not None and M_actual != self._committed_M:
            raise ValueError(
                f"Expected M={self._committed_M} (product of leading dims), got {M_actual}"
            )
        self.M = M_actual
        self.N = N
        self.dtype = expected_dtype
        self._affine_itemsize = weight.dtype.itemsize

        kernel = self._get_kernel(M_actual, N, expected_dtype, x.device.index)
        y, residual_out = kernel(x, residual, weight, bias)
        self._last_roofline_mn = (M_actual, N)
        return y.reshape(orig_shape), residual_out.reshape(orig_shape)
