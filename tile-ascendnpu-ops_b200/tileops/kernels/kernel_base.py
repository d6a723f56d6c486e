"""Kernel base class.

Mirrors the reference ``Kernel`` ABC
(examples/TileOPs/tileops/kernels/kernel_base.py:22-94): ``supported_archs``,
``default_config`` / ``init_config``, ``dtype_str`` and ``__call__ -> forward``.
A kernel here is a thin shim: ``forward`` validates nothing the op did not
already validate, allocates the outputs with torch (the caching allocator
owns all device memory) and launches one native entry point of
``libtileops_b200.so`` on the current torch stream.

``ascend_mode`` (the npuir programming mode of the reference) has no meaning
on CUDA; the attribute is kept for interface compatibility and ignored.
"""

from abc import ABC, abstractmethod
from typing import Any, Dict, Optional

import torch


class Kernel(ABC):
    """Abstract base class for native operator kernels."""

    dtype: Optional[torch.dtype] = None
    config: Dict[str, Any]
    # CUDA compute capabilities (major*10 + minor) the kernel runs on; the
    # library is built for sm_100a only.
    supported_archs: Optional[list] = [100]
    kernel: Optional[Any] = None
    ascend_mode: Optional[str] = None

    def __init__(self, *args: Any, **kwargs: Any) -> None:
        self.config = {}

    def init_config(self, config: Optional[Dict[str, Any]] = None) -> None:
        merged = dict(self.default_config)
        if config is not None:
            for k in merged:
                if config.get(k) is not None:
                    merged[k] = config[k]
        self.config = merged

    @property
    def dtype_str(self) -> str:
        """The dtype as its torch name (``"bfloat16"``)."""
        return self.dtype_to_str(self.dtype)

    @staticmethod
    def dtype_to_str(dtype: torch.dtype) -> str:
        return str(dtype).split(".")[-1]

    @property
    def default_config(self) -> Dict[str, Any]:
        return {}

    @abstractmethod
    def forward(self, *args: Any, **kwargs: Any) -> Any:
        raise NotImplementedError

    def __call__(self, *args: Any, **kwargs: Any) -> Any:
        return self.forward(*args, **kwargs)


def check_dtype(kernel: Kernel, dtype: torch.dtype, supported: tuple) -> None:
    """Raise the reference's kernel-level dtype error."""
    if dtype not in supported:
        names = ", ".join(str(dt) for dt in supported)
        raise ValueError(
            f"{kernel.__class__.__name__} only supports dtypes [{names}], got {dtype}"
        )
