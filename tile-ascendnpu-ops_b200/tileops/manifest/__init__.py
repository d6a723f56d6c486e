"""Op specs of the hot-path ops: workload shapes and roofline formulas.

Same loader interface as the reference (manifest/__init__.py:28-89):
``load_manifest()`` merges every ``*.yaml`` in this package (an op defined
twice is an error) and ``load_workloads(op_name)`` returns its workload rows.
"""

from __future__ import annotations

import functools
from pathlib import Path
from typing import Any

import yaml

_DIR = Path(__file__).resolve().parent
WORKLOAD_RESERVED_KEYS: frozenset[str] = frozenset({"dtypes", "label"})


def manifest_files() -> list[Path]:
    return sorted(_DIR.glob("*.yaml"))


@functools.lru_cache(maxsize=1)
def load_manifest() -> dict[str, Any]:
    merged: dict[str, Any] = {}
    origin: dict[str, str] = {}
    for path in manifest_files():
        ops = yaml.safe_load(path.read_text(encoding="utf-8")) or {}
        if not isinstance(ops, dict):
            raise ValueError(f"manifest file {path.name} must contain a top-level mapping")
        for name, entry in ops.items():
            if name in merged:
                raise ValueError(
                    f"duplicate op {name!r} in {path.name} (already defined in {origin[name]})"
                )
            merged[name] = entry
            origin[name] = path.name
    return merged


def load_workloads(op_name: str) -> list[dict[str, Any]]:
    ops = load_manifest()
    if op_name not in ops:
        raise KeyError(f"op '{op_name}' not found in ops manifest")
    return ops[op_name]["workloads"]
