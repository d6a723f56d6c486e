"""Op reconstruction helper kept at the reference's import path.

The reference runs its profiler in a subprocess that rebuilds each Op from
its constructor arguments (benchmark/msprof.py:108-139); tests assert that
contract through ``_extract_op_init_args``.  The Ascend profiler itself does
not exist on this platform; only the helper is provided.
"""

from __future__ import annotations

import inspect
from typing import Any

import torch

_SIMPLE = (bool, int, float, str, type(None), torch.dtype)


def _is_serializable(val: Any) -> bool:
    if isinstance(val, _SIMPLE):
        return True
    if isinstance(val, (tuple, list)):
        return all(_is_serializable(v) for v in val)
    return False


def _extract_op_init_args(op: Any) -> dict:
    """Constructor arguments of ``op``, read back from same-named attributes.

    Parameters of ``type(op).__init__`` (minus ``self`` and ``*args`` /
    ``**kwargs``) whose attribute exists on ``op`` and holds a simple value
    (numbers, strings, None, torch dtypes and tuples / lists of those).
    """
    try:
        sig = inspect.signature(type(op).__init__)
    except (ValueError, TypeError):
        return {}
    out: dict = {}
    for name, param in sig.parameters.items():
        if name == "self" or param.kind in (
            inspect.Parameter.VAR_POSITIONAL,
            inspect.Parameter.VAR_KEYWORD,
        ):
            continue
        if hasattr(op, name):
            val = getattr(op, name)
            if _is_serializable(val):
                out[name] = val
    return out
