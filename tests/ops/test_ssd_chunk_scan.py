"""SSDChunkScanFwdOp against the reference SSD golden.

The reference validates its kernel against golden_ssd_chunk_scan_fwd
(examples/TileOPs/tileops/kernels/mamba/ssd_chunk_scan/ssd_chunk_scan_kernel/
perf_opt/_ssd_chunk_scan_fwd_kernel.py:123-178) with |out - ref| <= atol +
1e-5 |ref| (atol 1e-3 fp16, 2e-3 bf16; :678-722) on its L0 / L1 / L2 /
boundary cases (:762-825) and a contract check (:732-758).  The same cases
run here against the oracle restatement, plus the committed fixtures of the
reference golden itself.
"""

import pytest
import torch

from oracle import reference as ref
from tests.golden.load import load, names
from tileops.ops.mamba import SSDChunkScanFwdOp

_ATOL = {torch.float16: 1e-3, torch.bfloat16: 2e-3}
_RTOL = 1e-5


def _inputs(B, C, Q, H, P, N, G, dtype, seed=0, decay=1.0):
    g = torch.Generator().manual_seed(seed)
    S = C * Q
    x = (torch.randn(B, S, H, P, generator=g) * 0.1).to(dtype)
    cb = (torch.randn(B, C, G, Q, Q, generator=g) * 0.1).to(dtype)
    dA = -torch.rand(B, H, C, Q, generator=g).cumsum(-1) * decay
    Cm = (torch.randn(B, S, G, N, generator=g) * 0.1).to(dtype)
    prev = torch.randn(B, C, H, P, N, generator=g) * 0.1
    dt = (torch.rand(B, H, C, Q, generator=g) * 0.1 + 0.01).to(dtype)
    return [t.cuda() for t in (x, cb, dA, Cm, prev, dt)]


def _gate(out, expect, dtype):
    diff = (out.cpu() - expect).abs()
    tol = _ATOL[dtype] + _RTOL * expect.abs()
    assert bool((diff <= tol).all()), f"max_diff {diff.max().item():.3e}"


def _case(B, C, Q, H, P, N, G, dtype, seed=0, decay=1.0):
    inp = _inputs(B, C, Q, H, P, N, G, dtype, seed, decay)
    out = SSDChunkScanFwdOp()(*inp)
    assert out.shape == (B, C * Q, H, P) and out.dtype == torch.float32 and out.is_contiguous()
    _gate(out, ref.ssd_chunk_scan(*inp, G), dtype)
    return out


@pytest.mark.gpu
@pytest.mark.parametrize("name", names("ssd_chunk_scan_"))
def test_golden_fixtures(name):
    case = load(name)
    i = case["inputs"]
    dtype = i["x"].dtype
    out = SSDChunkScanFwdOp()(*(i[n].cuda() for n in ("x", "cb", "dA_cumsum", "C",
                                                       "prev_states", "dt")))
    _gate(out, case["outputs"]["out"], dtype)


_L0 = [(1, 2, 64, 4, 64, 32, 1, torch.float16, 0), (1, 2, 128, 4, 128, 32, 1, torch.bfloat16, 1),
       (2, 4, 64, 8, 64, 64, 2, torch.float16, 2), (2, 2, 64, 4, 64, 32, 2, torch.bfloat16, 3),
       (1, 2, 96, 4, 48, 48, 1, torch.float16, 4),
       (1, 16, 256, 48, 64, 128, 1, torch.float16, 5),
       (1, 16, 256, 48, 64, 128, 1, torch.bfloat16, 6)]
_L1 = [(2, 4, 128, 8, 64, 64, 2, dt, 10 + i) for i, dt in enumerate((torch.float16, torch.bfloat16))] + \
      [(1, 16, 64, 48, 64, 64, 8, dt, 12 + i) for i, dt in enumerate((torch.float16, torch.bfloat16))] + \
      [(2, 8, 256, 8, 128, 128, 2, dt, 14 + i) for i, dt in enumerate((torch.float16, torch.bfloat16))]
_BOUNDARY = [(1, 2, 96, 4, 48, 48, 1, torch.bfloat16, 30), (1, 2, 64, 4, 64, 16, 1, torch.float16, 31),
             (1, 3, 64, 4, 64, 32, 1, torch.float16, 32), (1, 2, 80, 4, 64, 32, 1, torch.float16, 33)]


@pytest.mark.gpu
@pytest.mark.parametrize("B, C, Q, H, P, N, G, dtype, seed", _L0 + _L1 + _BOUNDARY)
def test_reference_cases(B, C, Q, H, P, N, G, dtype, seed):
    _case(B, C, Q, H, P, N, G, dtype, seed)


@pytest.mark.gpu
@pytest.mark.parametrize("B, C, Q, H, P, N, G, dtype, seed, decay", [
    (1, 1, 64, 4, 64, 32, 1, torch.float16, 20, 1.0),
    (4, 8, 64, 80, 128, 64, 8, torch.float16, 21, 1.0),
    (2, 4, 64, 8, 64, 64, 2, torch.bfloat16, 22, 100.0),
    (2, 2, 128, 4, 64, 64, 2, torch.float16, 23, 100.0),
])
def test_reference_l2_cases(B, C, Q, H, P, N, G, dtype, seed, decay):
    _case(B, C, Q, H, P, N, G, dtype, seed, decay)


@pytest.mark.gpu
@pytest.mark.parametrize("Q, N", [(200, 24), (136, 256), (320, 128), (1024, 64)])
def test_odd_chunk_and_state_sizes(Q, N):
    """Chunks that are not a multiple of 64 / 128 rows, d_state not a
    multiple of 16, the largest d_state and chunk length."""
    _case(1, 2, Q, 4, 64, N, 2, torch.bfloat16, seed=40 + N)


@pytest.mark.gpu
@pytest.mark.parametrize("key", [100, 64, 255])
def test_nan_decay_stays_in_its_rows(key):
    """A NaN in dA at key s of one (chunk, head) makes exactly rows l >= s of
    that chunk and head NaN, as the golden's masked decay does; rows before it
    and every other chunk / head keep their values.  bf16 with chunk 256 takes
    the kernel's scaled-x decay form, whose finiteness check must send the
    affected tiles to the per-block W build (a scaled x row of NaN would reach
    the rows above the diagonal too); key 64 is the first key of a block."""
    x, cb, dA, Cm, prev, dt = _inputs(1, 2, 256, 4, 64, 128, 1, torch.bfloat16, seed=50)
    dA = dA.cpu()
    dA[0, 1, 0, key] = float("nan")
    dA = dA.cuda()
    out = SSDChunkScanFwdOp()(x, cb, dA, Cm, prev, dt).cpu()
    expect = ref.ssd_chunk_scan(x, cb, dA, Cm, prev, dt, 1)
    nan_rows = torch.zeros(2 * 256, 4, dtype=torch.bool)
    nan_rows[key:256, 1] = True  # chunk 0, head 1, rows l >= key
    assert torch.equal(torch.isnan(expect).all(-1)[0], nan_rows)
    assert torch.equal(torch.isnan(out), torch.isnan(expect))
    keep = ~torch.isnan(expect)
    diff = (out[keep] - expect[keep]).abs()
    assert bool((diff <= _ATOL[torch.bfloat16] + _RTOL * expect[keep].abs()).all()), \
        f"max_diff {diff.max().item():.3e}"


@pytest.mark.gpu
def test_deterministic():
    inp = _inputs(1, 4, 128, 8, 64, 64, 1, torch.bfloat16, seed=7)
    op = SSDChunkScanFwdOp()
    assert torch.equal(op(*inp), op(*inp))


@pytest.mark.gpu
def test_contract_and_validation():
    op = SSDChunkScanFwdOp()
    with pytest.raises(RuntimeError, match="requires a prior forward"):
        op.eval_roofline()
    inp = _inputs(1, 2, 64, 4, 64, 32, 1, torch.float16)
    out = op(*inp)
    flops, nbytes = op.eval_roofline()
    tokens = 1 * 128 * 4
    assert flops == 2 * tokens * 32 * 64 + 1 * 2 * 4 * 64 * 64 * 64
    assert nbytes > 0 and out.shape == (1, 128, 4, 64)
    x, cb, dA, Cm, prev, dt = inp
    with pytest.raises(ValueError, match="x seq_len must equal"):
        op(x[:, :100], cb, dA, Cm, prev, dt)
    with pytest.raises(ValueError, match="cb must have shape"):
        op(x, cb[..., :32], dA, Cm, prev, dt)
    with pytest.raises(ValueError, match="prev_states must have shape"):
        op(x, cb, dA, Cm, prev[..., :16], dt)
    with pytest.raises(ValueError, match="n_heads must be divisible by n_groups"):
        Cm3 = torch.zeros(1, 128, 3, 32, dtype=torch.float16, device="cuda")
        op(x, cb, dA, Cm3, prev, dt)
    with pytest.raises(ValueError, match="x must be a cuda tensor"):
        op(x.cpu(), cb, dA, Cm, prev, dt)
    with pytest.raises(ValueError, match="cb.dtype"):
        op(x, cb.bfloat16(), dA, Cm, prev, dt)


@pytest.mark.gpu
@pytest.mark.parametrize("Q, P, N, G, dtype", [
    (100, 16, 8, 1, torch.bfloat16),    # chunk not a multiple of 8: element cb loads
    (72, 32, 24, 2, torch.float16),
    (130, 128, 256, 1, torch.bfloat16),  # largest head and state, a 2-row second tile
])
def test_small_and_ragged_dims(Q, P, N, G, dtype):
    _case(2, 3, Q, 4, P, N, G, dtype, seed=50 + Q)
