"""Base classes for workload definitions shared by tests and benchmarks.

Same contract as the reference (workloads/workload_base.py:20-61):
``WorkloadBase.gen_inputs()``, ``RandnWorkload(shape, dtype)`` drawing one
``torch.randn`` tensor on the backend device, and ``FixtureBase`` whose
subclasses are usable as ``@Fixture`` decorators that apply their ``PARAMS``
(or ``get_params()``) as ``pytest.mark.parametrize``.
"""

from __future__ import annotations

from abc import ABC, abstractmethod
from typing import Any, Callable, TypeVar

import torch

from tileops.device import get_device_backend

_F = TypeVar("_F", bound=Callable[..., Any])


class WorkloadBase(ABC):
    """Input generation plus parameters."""

    @abstractmethod
    def gen_inputs(self) -> tuple[Any, ...]:
        raise NotImplementedError


class RandnWorkload(WorkloadBase):
    """One ``torch.randn`` tensor of ``shape`` / ``dtype`` on the device."""

    def __init__(self, shape: tuple, dtype: torch.dtype):
        self.shape = shape
        self.dtype = dtype

    def gen_inputs(self) -> tuple[torch.Tensor]:
        device = get_device_backend().name
        return (torch.randn(*self.shape, dtype=self.dtype, device=device),)


class FixtureMeta(type):
    """Makes Fixture subclasses usable as decorators."""

    def __call__(cls, fn: _F) -> _F:
        import pytest

        params = cls.get_params() if hasattr(cls, "get_params") else cls.PARAMS
        for names, values in reversed(params):
            fn = pytest.mark.parametrize(names, values)(fn)
        return fn


class FixtureBase(metaclass=FixtureMeta):
    """Base class for reusable parametrize decorators."""

    PARAMS = []
