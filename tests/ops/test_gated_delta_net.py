"""GPU parity of GatedDeltaNetPrefillFwdOp against the sequential golden.

The reference has no test for this op; its only pin is the probe's
sequential golden (examples/gdn_prefill/probe/gdn_prefill_probe.py:60-77),
restated in the oracle and checked bit-for-bit against fixtures of it.  The
kernel runs the chunked WY form with bf16 tensor-core operands and an fp32
state; o is compared against the fp32 golden with the north-star 16-bit
tolerance (atol = rtol = 1e-2), the fp32 final state with the bound measured
against an fp64 recurrence (STATE_TOL below).
Covered: the probe's own cases at the supported head dims, BASELINE
distributions at small sizes, ragged lengths (T not a multiple of 64),
initial-state chaining (two halves == one run), dk = dv = 64, and the
BASELINE (4, 8192, 16, 128) configuration on sampled (batch, head) pairs.
"""

import pytest
import torch

from oracle import reference as ref
from tests.golden.load import load
from tileops.ops.linear_attention import GatedDeltaNetPrefillFwdOp
from tileops.workloads.linear_attention import GdnPrefillWorkload

pytestmark = pytest.mark.gpu

TOL = dict(atol=1e-2, rtol=1e-2)  # the bf16 output o: the north-star 16-bit tolerance
# The fp32 final state: the state enters the tensor cores in bf16 each chunk
# (S as the B operand of Wk S and Q S; err and the decayed err in bf16), so
# fp32's 1e-5 is out of reach.  Measured against an fp64 recurrence on the
# BASELINE distributions (B=4, T=8192, H=16, and every shape of this file):
# max |error| 2.4e-3 to 4.7e-3 at |S| <= 0.93, within atol 3.8e-3 + rtol 1e-3;
# the bound keeps a 2x margin.
STATE_TOL = dict(atol=8e-3, rtol=1e-3)


def _run(q, k, v, g, beta, h0=None):
    b, t, h, dk = q.shape
    op = GatedDeltaNetPrefillFwdOp(b, t, h, dk, v.shape[-1], dtype=q.dtype)
    return op(q, k, v, g, beta, h0)


def _check(q, k, v, g, beta, h0=None):
    o, s = _run(q, k, v, g, beta, h0)
    o_ref, s_ref = ref.gdn_prefill_bthd(q, k, v, g, beta, None, h0)
    torch.testing.assert_close(o.cpu().float(), o_ref.float(), **TOL)
    torch.testing.assert_close(s.cpu(), s_ref, **STATE_TOL)
    return o, s


@pytest.mark.parametrize("name", ["gdn_b1_h1_t192_d64_dv64", "gdn_b1_h1_t130_d128_dv128"])
def test_probe_cases(name):
    """The probe's input distributions (fp16 there, bf16 here) and initial state."""
    case = load(name)
    i = case["inputs"]
    t = lambda a: a.transpose(1, 2).contiguous().cuda()  # noqa: E731  BHTD -> BTHD
    q, k, v = (t(i[n]).to(torch.bfloat16) for n in ("q", "k", "v"))
    g, beta = t(i["g"]).float(), t(i["beta"]).float()
    _check(q, k, v, g, beta, i["state0"].cuda())


@pytest.mark.parametrize("batch, seq_len, heads, dk, dv", [
    (1, 64, 1, 128, 128), (2, 512, 2, 128, 128), (1, 1000, 2, 128, 128),
    (2, 256, 3, 64, 64), (1, 320, 2, 128, 64), (1, 192, 1, 64, 128),
])
def test_baseline_distributions(batch, seq_len, heads, dk, dv):
    _check(*GdnPrefillWorkload(batch, seq_len, heads, dk, dv).gen_inputs())


@pytest.mark.parametrize("seq_len", [1, 5, 63, 65, 127, 129])
def test_ragged_lengths(seq_len):
    _check(*GdnPrefillWorkload(1, seq_len, 2, 128, 128).gen_inputs())


def test_initial_state_chaining():
    q, k, v, g, beta = GdnPrefillWorkload(1, 384, 2, 128, 128).gen_inputs()
    o_full, s_full = _run(q, k, v, g, beta)
    cut = 256
    o1, s1 = _run(q[:, :cut], k[:, :cut], v[:, :cut], g[:, :cut], beta[:, :cut])
    o2, s2 = _run(q[:, cut:], k[:, cut:], v[:, cut:], g[:, cut:], beta[:, cut:], s1)
    torch.testing.assert_close(torch.cat([o1, o2], 1).float(), o_full.float(), atol=2e-3,
                               rtol=2e-3)
    torch.testing.assert_close(s2, s_full, atol=1e-4, rtol=1e-4)


def test_deterministic():
    inputs = GdnPrefillWorkload(2, 256, 2, 128, 128).gen_inputs()
    o0, s0 = _run(*inputs)
    o1, s1 = _run(*inputs)
    assert torch.equal(o0, o1) and torch.equal(s0, s1)


def test_roofline_formula():
    op = GatedDeltaNetPrefillFwdOp(4, 8192, 16, 128, 128)
    flops, nbytes = op.eval_roofline()
    assert flops == 4 * 8192 * 16 * 155_648
    assert nbytes == 4 * 134_217_728 + 2 * 2_097_152 + 4_194_304


def test_rejects_bad_inputs():
    q, k, v, g, beta = GdnPrefillWorkload(1, 64, 1, 128, 128).gen_inputs()
    op = GatedDeltaNetPrefillFwdOp(1, 64, 1, 128, 128)
    with pytest.raises(ValueError, match="q.shape"):
        op(q[:, :32], k, v, g, beta)
    with pytest.raises(ValueError, match="v.dtype"):
        op(q, k, v.half(), g, beta)
    with pytest.raises(ValueError, match="dim_k"):
        GatedDeltaNetPrefillFwdOp(1, 64, 1, 96, 128)


@pytest.mark.full
def test_baseline_config_sampled_heads():
    """BASELINE: B=4, T=8192, H=16, dk=dv=128; (b, h) pairs checked against the golden."""
    q, k, v, g, beta = GdnPrefillWorkload(4, 8192, 16, 128, 128).gen_inputs()
    o, s = _run(q, k, v, g, beta)
    for bi, hi in ((0, 0), (3, 15)):
        sl = (slice(bi, bi + 1), slice(None), slice(hi, hi + 1))
        o_ref, s_ref = ref.gdn_prefill_bthd(q[sl], k[sl], v[sl], g[sl], beta[sl])
        torch.testing.assert_close(o[sl].cpu().float(), o_ref.float(), **TOL)
        torch.testing.assert_close(s[bi : bi + 1, hi : hi + 1].cpu(), s_ref, **STATE_TOL)


def test_misaligned_final_state_runs_the_register_scan():
    """dk = 128 normally scans on tcgen05, which stores the final state with
    16-byte vectors; a final_state pointer off that alignment runs the
    mma.sync register scan instead.  Both must match the golden."""
    from tileops import _native as nat

    q, k, v, g, beta = GdnPrefillWorkload(1, 320, 2, 128, 128).gen_inputs()
    B, T, H, DK = q.shape
    DV = v.shape[-1]
    nbytes = nat.lib().tileops_gdn_workspace_bytes(B, T, H, DK, DV)
    ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    o = torch.empty_like(v)
    buf = torch.zeros(B * H * DK * DV + 1, dtype=torch.float32, device="cuda")
    hT = buf[1:]  # 4 bytes past a 16-byte boundary
    nat.launch("tileops_gdn_prefill_fwd", q.device, nat.ptr(q), nat.ptr(k), nat.ptr(v),
               nat.ptr(g), nat.ptr(beta), nat.ptr(None), nat.ptr(o), nat.ptr(hT), nat.ptr(ws),
               B, T, H, DK, DV, 64, DK ** -0.5, nat.dtype_code(torch.bfloat16))
    torch.cuda.synchronize()
    o_ref, s_ref = ref.gdn_prefill_bthd(q, k, v, g, beta)
    torch.testing.assert_close(o.cpu().float(), o_ref.float(), **TOL)
    torch.testing.assert_close(hT.view(B, H, DK, DV).cpu(), s_ref, **STATE_TOL)
    o_tc, s_tc = _run(q, k, v, g, beta)
    torch.testing.assert_close(o.float(), o_tc.float(), atol=2e-2, rtol=2e-2)


def test_strong_decay_takes_the_exact_exponentials():
    """A chunk whose cumulative log-decay passes -80 forms e^(gc_l - gc_s) per
    entry instead of e^gc_l * e^-gc_s (whose factors would overflow fp32);
    chunks of both kinds in one call."""
    q, k, v, g, beta = GdnPrefillWorkload(1, 256, 2, 128, 128).gen_inputs()
    g = g.clone()
    g[:, 64:128] = -2.5  # the second chunk reaches gc = -160
    _check(q, k, v, g, beta)
