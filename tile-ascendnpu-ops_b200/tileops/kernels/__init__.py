from tileops.kernels.kernel_base import Kernel

__all__ = ["Kernel"]
