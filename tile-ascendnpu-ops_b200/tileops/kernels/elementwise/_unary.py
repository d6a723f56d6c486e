"""Shared shim for the flat elementwise kernels (one input, one output).

The reference kernels (e.g. kernels/elementwise/hardswish/hardswish.py:82-...)
take ``(N_total, dtype, config=None)``, check the dtype against the manifest
list with the message ``"<Kernel> only supports dtypes [...]"``, and their
``forward(x)`` maps a contiguous 1-D tensor of ``N_total`` elements to a new
tensor.  Here ``forward`` allocates the output and launches the matching
``tileops_*_fwd`` entry point.
"""

from typing import Optional

import torch

from tileops import _native
from tileops.kernels.kernel_base import Kernel, check_dtype

FLOAT_DTYPES = (torch.float16, torch.bfloat16, torch.float32)


class UnaryNativeKernel(Kernel):
    """Flat unary kernel over ``N_total`` elements."""

    SUPPORTED_DTYPES: tuple = FLOAT_DTYPES
    entry_point: str = ""
    bool_output: bool = False

    def __init__(self, N_total: int, dtype: torch.dtype, config: Optional[dict] = None):
        super().__init__()
        check_dtype(self, dtype, self.SUPPORTED_DTYPES)
        self.N_total = int(N_total)
        self.dtype = dtype
        self.output_dtype = torch.bool if self.bool_output else dtype
        self.init_config(config)

    def _scalar_args(self) -> tuple:
        return ()

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x = x.contiguous()
        y = torch.empty(x.shape, dtype=self.output_dtype, device=x.device)
        _native.launch(
            self.entry_point,
            x.device,
            _native.ptr(x),
            _native.ptr(y),
            x.numel(),
            _native.dtype_code(self.dtype),
            *self._scalar_args(),
        )
        return y
