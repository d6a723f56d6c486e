"""Op base class.

Same interface as the reference ``Op``
(examples/TileOPs/tileops/ops/op_base.py:31-119): ``default_kernel_map``,
``dispatch_kernel`` (resolve a ``kernel_map`` override against the defaults
and check the kernel's ``supported_archs``), ``forward``, ``__call__``,
``eval_roofline`` and ``_cache_key``.  The architecture check compares CUDA
compute capabilities; it is skipped when no GPU is present so ops can be
constructed (and their roofline formulas evaluated) on a CPU-only host.
"""

from __future__ import annotations

import warnings
from abc import ABC, abstractmethod
from typing import Hashable, Optional, Union

import torch

from tileops.device import get_device_backend
from tileops.kernels.kernel_base import Kernel


class Op(ABC):
    """Base class of every ``*FwdOp``."""

    kernel: Optional[Kernel] = None
    kernel_map: Optional[dict[str, Kernel]] = None
    dtype: Optional[torch.dtype] = None
    input_shapes: Optional[list[tuple]] = None
    _static_axes: frozenset[tuple[int, int]] = frozenset()

    @property
    @abstractmethod
    def default_kernel_map(self) -> dict[str, Kernel]:
        raise NotImplementedError("Op must implement default_kernel_map")

    def _install_kernel_map(self, candidate_map: Optional[dict[str, Kernel]] = None) -> None:
        default_map = self.default_kernel_map
        if not default_map:
            self.kernel_map = dict(candidate_map) if candidate_map else {}
            return
        resolved: dict[str, Kernel] = {}
        backend = get_device_backend()
        for name, default_kernel in default_map.items():
            kernel_type = (
                candidate_map[name]
                if candidate_map is not None and name in candidate_map
                else default_kernel
            )
            if (
                kernel_type is not None
                and kernel_type.supported_archs is not None
                and not _arch_supported(kernel_type.supported_archs, backend)
            ):
                raise ValueError(
                    f"{kernel_type.__name__} is not supported on backend "
                    f"{backend.name} (supported: {kernel_type.supported_archs})"
                )
            resolved[name] = kernel_type
        self.kernel_map = resolved

    def dispatch_kernel(self, kernel_map: Optional[dict[str, Kernel]] = None) -> None:
        """Resolve and install the kernel map."""
        self._install_kernel_map(kernel_map)

    @abstractmethod
    def forward(self, *args: object, **kwargs: object) -> Union[torch.Tensor, tuple]:
        raise NotImplementedError("forward method is not implemented")

    def __call__(self, *args: object, **kwargs: object) -> Union[torch.Tensor, tuple]:
        return self.forward(*args, **kwargs)

    def eval_roofline(self) -> tuple[int, int]:
        """Return ``(flops, bytes)`` for this op instance."""
        raise NotImplementedError(
            f"{type(self).__name__}.eval_roofline() must be implemented by the concrete Op."
        )

    def _cache_key(self, *input_shapes: tuple[int, ...]) -> Hashable:
        """Cache key for kernel dispatch given forward-time input shapes."""
        if not self._static_axes and type(self)._cache_key is Op._cache_key:
            warnings.warn(
                f"{type(self).__name__}: Op._cache_key() called with empty _static_axes "
                f"and no subclass override.",
                stacklevel=2,
            )
        return tuple(
            s
            for i, shape in enumerate(input_shapes)
            for axis, s in enumerate(shape)
            if (i, axis) not in self._static_axes
        )


def _arch_supported(supported: list, backend: object) -> bool:
    """True when the current GPU's compute capability is in ``supported``.

    Without a GPU nothing can launch anyway; construction is allowed so that
    host-side logic (validation, roofline formulas) stays testable.
    """
    if supported is None or not backend.is_available():
        return True
    major, minor = torch.cuda.get_device_capability()
    return (major * 10 + minor) in supported or major * 10 in supported
