"""The device backend: CUDA only.

The reference funnels every device call through a ``DeviceBackend``
singleton with NPU, CUDA and CPU implementations detected in that order
(examples/TileOPs/tileops/device.py:37-103, :227-316, :374-393).  This build
targets one device, the B200, so there is exactly one backend.  It keeps the
reference's interface (``name``, ``is_device_tensor``, ``Event``,
``synchronize``, ``cache_flush``, ``shared_memory_budget`` …) so the op layer,
tests and benchmarks read the same; ``name`` is always ``"cuda"``, which is
also what the ops' "must be a cuda tensor" errors print.

Nothing here falls back to the CPU: on a machine without a GPU the backend
reports ``is_available() == False`` and any kernel call raises.
"""

from __future__ import annotations

from typing import Optional

import torch

__all__ = ["CUDABackend", "DeviceBackend", "get_device_backend", "reset_device_backend"]


class CUDABackend:
    """NVIDIA CUDA backend (B200, sm_100a)."""

    name = "cuda"

    def is_available(self) -> bool:
        return torch.cuda.is_available()

    def device_count(self) -> int:
        return torch.cuda.device_count()

    def current_device(self) -> int:
        return torch.cuda.current_device()

    def synchronize(self, device: Optional[int] = None) -> None:
        torch.cuda.synchronize(device)

    def empty_cache(self) -> None:
        torch.cuda.empty_cache()

    def get_device_name(self, device: Optional[int] = None) -> str:
        return torch.cuda.get_device_name(device) if self.is_available() else ""

    def get_device_properties(self, device: Optional[int] = None) -> object:
        return torch.cuda.get_device_properties(device)

    def is_device_tensor(self, tensor: torch.Tensor) -> bool:
        return isinstance(tensor, torch.Tensor) and tensor.is_cuda

    def Event(self, enable_timing: bool = False) -> object:  # noqa: N802 (reference name)
        return torch.cuda.Event(enable_timing=enable_timing)

    def manual_seed_all(self, seed: int) -> None:
        torch.manual_seed(seed)
        if self.is_available():
            torch.cuda.manual_seed_all(seed)

    def supports_profiler(self) -> bool:
        return True

    def shared_memory_budget(self, device: Optional[int] = None) -> int:
        """Opt-in shared memory per block (227 KiB on B200)."""
        if not self.is_available():
            if device is not None:
                raise RuntimeError(f"CUDA is not available but device={device} was requested")
            return 48 * 1024
        props = torch.cuda.get_device_properties(
            torch.cuda.current_device() if device is None else device
        )
        return int(getattr(props, "shared_memory_per_block_optin", 0) or 48 * 1024)

    _l2_flush_cache: Optional[torch.Tensor] = None

    def cache_flush(self) -> None:
        """Evict L2 by zeroing a buffer twice its size (126 MB L2 on B200)."""
        if self._l2_flush_cache is None:
            l2 = torch.cuda.get_device_properties(torch.cuda.current_device()).L2_cache_size
            nbytes = 2 * (l2 if l2 > 0 else 128 * 1024 * 1024)
            self._l2_flush_cache = torch.empty(nbytes // 4, dtype=torch.int32, device="cuda")
        self._l2_flush_cache.zero_()

    def env_metadata(self) -> list[str]:
        lines = [
            f"- **Torch version**: {torch.__version__}",
            f"- **CUDA version (torch)**: {torch.version.cuda or 'N/A'}",
        ]
        lines.append(
            f"- **GPU model**: {self.get_device_name(0)}"
            if self.is_available()
            else "- **GPU model**: N/A (no CUDA device)"
        )
        return lines


# The reference's abstract base is named DeviceBackend; with one backend the
# name is an alias kept for imports.
DeviceBackend = CUDABackend

_backend: Optional[CUDABackend] = None


def get_device_backend() -> CUDABackend:
    """Return the process-wide backend singleton."""
    global _backend
    if _backend is None:
        _backend = CUDABackend()
    return _backend


def reset_device_backend() -> None:
    """Drop the cached backend (tests)."""
    global _backend
    _backend = None


DEFAULT_DEVICE: str = "cuda"
