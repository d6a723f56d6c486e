"""Load the committed golden fixtures (written by make_golden.py)."""

from pathlib import Path

import torch

DIR = Path(__file__).resolve().parent


def names(prefix: str = "") -> list[str]:
    return sorted(p.stem for p in DIR.glob(f"{prefix}*.pt"))


def load(name: str) -> dict:
    return torch.load(DIR / f"{name}.pt", weights_only=False)
