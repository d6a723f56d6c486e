"""Small helpers shared by ops and workloads."""

import torch

_STR2DTYPE = {
    "float32": torch.float32,
    "float16": torch.float16,
    "bfloat16": torch.bfloat16,
    "bool": torch.bool,
    "uint8": torch.uint8,
    "int8": torch.int8,
    "int16": torch.int16,
    "int32": torch.int32,
    "int64": torch.int64,
}


def str2dtype(name: str) -> torch.dtype:
    """Map a manifest dtype name (``"bfloat16"``) to the torch dtype."""
    try:
        return _STR2DTYPE[name]
    except KeyError:
        raise ValueError(f"unknown dtype name {name!r}") from None
