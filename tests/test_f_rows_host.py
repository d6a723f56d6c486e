"""Host-side contracts of the GLA decode, SSD chunk scan and GDN varlen ops
(no GPU): constructor validation, scale resolution, kernel-cache keys and the
errors raised before any launch."""

import pytest
import torch

from tileops.kernels.linear_attention.gla_decode import GLADecodeKernel, _ceil_ktile_fit
from tileops.kernels.mamba import SSDChunkScanFwdKernel
from tileops.ops.linear_attention import GatedDeltaNetPrefillFwdOp, GLADecodeOp
from tileops.ops.mamba import SSDChunkScanFwdOp


def test_gla_scale_and_ktile():
    assert GLADecodeOp(1, 2, 64, 64).kernel.scale == pytest.approx(64 ** -0.5)
    assert GLADecodeOp(1, 2, 64, 64, scale=0.3).kernel.scale == pytest.approx(0.3)
    k = GLADecodeKernel(1, 1, 128, 128)
    assert k.config == {"k_tile": _ceil_ktile_fit(128, 128)} and 128 % k.k_tile == 0
    with pytest.raises(ValueError, match="divisible by k_tile"):
        GLADecodeKernel(1, 1, 96, 64, k_tile=64)


def test_gla_rejects_cpu_tensors():
    op = GLADecodeOp(1, 1, 16, 16, dtype=torch.float32)
    t = torch.zeros(1, 1, 16)
    with pytest.raises(ValueError, match="must be a"):
        op(t, t, t, t, torch.zeros(1, 1, 16, 16))


def test_ssd_kernel_validation():
    with pytest.raises(ValueError, match="only supports dtypes"):
        SSDChunkScanFwdKernel(1, 1, 64, 4, 64, 32, 1, torch.float32)
    with pytest.raises(ValueError, match="divisible by n_groups"):
        SSDChunkScanFwdKernel(1, 1, 64, 6, 64, 32, 4, torch.float16)
    with pytest.raises(ValueError, match="d_head"):
        SSDChunkScanFwdKernel(1, 1, 64, 4, 40, 32, 1, torch.float16)
    with pytest.raises(ValueError, match="d_state"):
        SSDChunkScanFwdKernel(1, 1, 64, 4, 64, 20, 1, torch.float16)
    with pytest.raises(ValueError, match="chunk_len"):
        SSDChunkScanFwdKernel(1, 1, 2048, 4, 64, 32, 1, torch.float16)
    k = SSDChunkScanFwdKernel(1, 2, 64, 4, 64, 32, 1, torch.bfloat16)
    assert k.config == {"block_l": 64, "block_p": 64, "block_n": 32, "block_s": 64,
                        "num_stages": 2}


def test_ssd_op_contract_without_gpu():
    op = SSDChunkScanFwdOp()
    with pytest.raises(RuntimeError, match="requires a prior forward"):
        op.eval_roofline()
    x = torch.zeros(1, 128, 4, 64, dtype=torch.float16)
    with pytest.raises(ValueError, match="x must be a"):
        op(x, None, None, None, None, None)


def test_gdn_varlen_argument_checks_without_gpu():
    op = GatedDeltaNetPrefillFwdOp(1, 64, 1, 128, 128)
    q = torch.zeros(1, 64, 1, 128, dtype=torch.bfloat16)
    g = torch.zeros(1, 64, 1)
    with pytest.raises(ValueError, match="must be a"):
        op(q, q, q, g, g, cu_seqlens=torch.tensor([0, 64], dtype=torch.int32))


def test_gla_manifest_rows_and_roofline():
    """Every GLADecodeOp manifest row builds an op whose eval_roofline is the
    manifest formula (reference linear_attention.yaml GLADecodeOp roofline)."""
    from tileops.manifest import load_manifest, load_workloads

    assert "SSDChunkScanFwdOp" in load_manifest()
    rows = load_workloads("GLADecodeOp")
    assert rows
    for row in rows:
        for dt in row["dtypes"]:
            dtype = getattr(torch, dt)
            b, h, dk, dv = row["B"], row["H"], row["DK"], row["DV"]
            flops, nbytes = GLADecodeOp(b, h, dk, dv, row["scale"], dtype).eval_roofline()
            assert flops == b * h * (5 * dk * dv + dk + dv)
            assert nbytes == b * h * (3 * dk + 2 * dv + 2 * dk * dv) * dtype.itemsize
