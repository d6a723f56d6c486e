"""Correctness-test base: run the op, compare with a reference program.

Same contract as the reference harness
(examples/TileOPs/tileops/testing/test_base.py:34-144): ``TestBase.check(op,
*inputs, compare=None, atol, rtol)`` runs ``ref_program`` first (an
out-of-memory there becomes a logged skip), then ``op(*inputs)`` under
``torch.no_grad()``, records the max absolute error for the pytest report
hook, and applies ``allclose_compare`` (``torch.testing.assert_close`` with
``equal_nan=True``) or a caller-supplied comparator per output; a ``None``
reference output is not checked.  Reference outputs computed on the CPU are
moved to the op output's device before comparing.
"""

from __future__ import annotations

import logging
from abc import abstractmethod
from functools import partial
from typing import Any

import torch

from tileops.workloads.workload_base import WorkloadBase

_logger = logging.getLogger("tileops.testing")


def _to_tuple(outputs):
    if isinstance(outputs, torch.Tensor):
        return (outputs,)
    if isinstance(outputs, (list, tuple)):
        return tuple(outputs)
    raise ValueError(f"Unsupported output type: {type(outputs)}")


def allclose_compare(output: torch.Tensor, output_ref: torch.Tensor, atol: float = 1e-8,
                     rtol: float = 1e-5) -> None:
    output_ref = output_ref.to(output.device)
    output, output_ref = torch.broadcast_tensors(output, output_ref)
    torch.testing.assert_close(output, output_ref, atol=atol, rtol=rtol, equal_nan=True)


def exact_compare(output: torch.Tensor, output_ref: torch.Tensor) -> None:
    assert torch.equal(output, output_ref.to(output.device)), (
        "output does not exactly match reference"
    )


class _CheckResult:
    """Last check's metadata, read by the conftest report hook."""

    op_name: str | None = None
    op_module: str | None = None
    max_abs_err: float | None = None


_check_result = _CheckResult()


def get_check_result() -> _CheckResult:
    return _check_result


def record_check_result(op, outputs: Any, outputs_ref: Any) -> float:
    """Record the op identity and the max absolute error over all outputs."""
    outputs = _to_tuple(outputs)
    outputs_ref = _to_tuple(outputs_ref)
    assert len(outputs) == len(outputs_ref), (
        f"outputs: {len(outputs)} and outputs_ref: {len(outputs_ref)} have different size"
    )
    max_abs_err = 0.0
    for output, output_ref in zip(outputs, outputs_ref, strict=True):
        if output_ref is not None:
            a = output.to(torch.float32)
            b = output_ref.to(device=output.device, dtype=torch.float32)
            diff = (a - b).abs()
            # NaN-equal positions (both NaN) and equal infinities carry no error.
            same = (a == b) | (torch.isnan(a) & torch.isnan(b))
            diff = torch.where(same, torch.zeros_like(diff), diff)
            if diff.numel():
                max_abs_err = max(max_abs_err, diff.max().item())
    _check_result.op_name = op.__class__.__name__
    _check_result.op_module = op.__class__.__module__
    _check_result.max_abs_err = max_abs_err
    return max_abs_err


class TestBase(WorkloadBase):
    """Op correctness test: subclasses provide ``gen_inputs`` and ``ref_program``."""

    __test__ = False

    @abstractmethod
    def ref_program(self, *inputs: Any) -> Any:
        raise NotImplementedError

    def check(self, op, *inputs: torch.Tensor, compare=None, atol: float = 1e-08,
              rtol: float = 1e-05) -> None:
        if compare is None:
            compare = partial(allclose_compare, atol=atol, rtol=rtol)
        op_name = op.__class__.__name__
        op_module = op.__class__.__module__
        try:
            outputs_ref = self.ref_program(*inputs)
        except RuntimeError as e:
            if "out of memory" in str(e):
                _logger.warning("op=%s module=%s status=skip_oom", op_name, op_module)
                return
            raise
        outputs_ref = _to_tuple(outputs_ref)
        with torch.no_grad():
            outputs = _to_tuple(op(*inputs))
        max_abs_err = record_check_result(op, outputs, outputs_ref)
        comparators = [compare] * len(outputs) if callable(compare) else list(compare)
        for output, output_ref, cmp in zip(outputs, outputs_ref, comparators, strict=True):
            if output_ref is not None:
                cmp(output, output_ref)
        _logger.info("op=%s module=%s status=pass max_abs_err=%.2e", op_name, op_module,
                     max_abs_err)
