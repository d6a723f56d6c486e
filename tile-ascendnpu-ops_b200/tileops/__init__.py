"""TileOPs forward operators on NVIDIA B200 (sm_100a).

A drop-in for the ``tileops`` package of Yihuace/tile-ascendnpu-ops
(``examples/TileOPs/tileops``): the same ``tileops.ops.*FwdOp`` classes,
constructor arguments, ``forward`` signatures, output tuples, error messages
and ``eval_roofline`` formulas, with every kernel a hand-written CUDA kernel
for sm_100a in ``libtileops_b200.so`` (C ABI: ``include/tileops_c.h``).

Layers (as in the reference):

    manifest  -- op specs and workload shapes (YAML)
    workloads -- seeded input generators shared by tests and benchmarks
    ops       -- Op ABC: validation, reshape, kernel dispatch, roofline
    kernels   -- Kernel ABC: thin shims over the C ABI
    testing   -- TestBase: correctness against a CPU reference
    benchmark -- CUDA-event latency with an L2 flush, roofline figures
    device    -- the CUDA device backend
"""

from tileops.device import get_device_backend

__all__ = ["get_device_backend"]
