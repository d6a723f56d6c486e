"""Pin the CPU oracle to the reference: oracle(fixture inputs) == fixture outputs.

The fixtures under tests/golden were computed by the reference's own ref
programs and golden functions (tests/golden/make_golden.py).  The oracle is
a restatement, so it must reproduce them bit for bit (NaN positions equal).
CPU only.
"""

import pytest
import torch

from oracle import reference as ref
from tests.golden.load import load, names


def assert_same(out: torch.Tensor, expect: torch.Tensor) -> None:
    assert out.dtype == expect.dtype and out.shape == expect.shape
    if out.dtype.is_floating_point:
        torch.testing.assert_close(out, expect, atol=0, rtol=0, equal_nan=True)
    else:
        assert torch.equal(out, expect)


@pytest.mark.parametrize("name", names("hardswish_") + names("hardsigmoid_"))
def test_oracle_unary(name):
    case = load(name)
    fn = ref.hardswish if name.startswith("hardswish") else ref.hardsigmoid
    assert_same(fn(case["inputs"]["x"]), case["outputs"]["y"])


@pytest.mark.parametrize("name", names("clamp_scalar_"))
def test_oracle_clamp_scalar(name):
    case = load(name)
    m = case["meta"]
    assert_same(ref.clamp_scalar(case["inputs"]["x"], m["min"], m["max"]), case["outputs"]["y"])


@pytest.mark.parametrize("name", names("clamp_min_"))
def test_oracle_clamp_min(name):
    case = load(name)
    assert_same(ref.clamp_min(case["inputs"]["x"], case["meta"]["min"]), case["outputs"]["y"])


@pytest.mark.parametrize("name", names("isnan_") + names("isinf_") + names("isfinite_"))
def test_oracle_predicates(name):
    case = load(name)
    fn = {"isnan": ref.isnan, "isinf": ref.isinf, "isfinite": ref.isfinite}[name.split("_")[0]]
    assert_same(fn(case["inputs"]["x"]), case["outputs"]["y"])


@pytest.mark.parametrize("name", names("bitwise_not_"))
def test_oracle_bitwise_not(name):
    case = load(name)
    assert_same(ref.bitwise_not(case["inputs"]["x"]), case["outputs"]["y"])


@pytest.mark.parametrize("name", names("gelu_and_mul_") + names("gelu_tanh_and_mul_"))
def test_oracle_gated(name):
    case = load(name)
    x = case["inputs"]["x"]
    if name.startswith("gelu_tanh"):
        assert_same(ref.gelu_tanh_and_mul(x), case["outputs"]["y"])
    elif "golden" in name:
        # golden_gelu_and_mul uses F.gelu (exact erf form); the oracle writes
        # the erf formula out, as the reference test does: equal within fp32 rounding.
        torch.testing.assert_close(ref.gelu_and_mul(x), case["outputs"]["y"], atol=1e-6,
                                   rtol=1e-6)
    else:
        assert_same(ref.gelu_and_mul(x), case["outputs"]["y"])


@pytest.mark.parametrize("name", names("fused_add_layer_norm_"))
def test_oracle_fused_add_layer_norm(name):
    case = load(name)
    i = case["inputs"]
    y, added = ref.fused_add_layer_norm(i["x"], i["residual"], i["weight"], i["bias"],
                                        case["meta"]["eps"])
    assert_same(y, case["outputs"]["y"])
    assert_same(added, case["outputs"]["residual_out"])


@pytest.mark.parametrize("name", [n for n in names("conv1d_") if "golden" not in n])
def test_oracle_conv1d(name):
    case = load(name)
    m, i = case["meta"], case["inputs"]
    y = ref.conv1d(i["x"], i["weight"], i["bias"], stride=m["stride"], padding=m["padding"],
                   dilation=m["dilation"], groups=m["groups"])
    assert_same(y, case["outputs"]["y"])


def test_oracle_causal_conv_matches_reference_depthwise_golden():
    case = load("conv1d_depthwise_golden_causal_bf16")
    i = case["inputs"]
    length = i["x"].shape[-1]
    y = ref.causal_depthwise_conv1d(i["x"], i["weight"], i["bias"])
    assert_same(y, case["outputs"]["y_full"][..., :length].contiguous())


@pytest.mark.parametrize("name", names("mha_"))
def test_oracle_mha(name):
    case = load(name)
    i, m = case["inputs"], case["meta"]
    o, lse = ref.gqa_prefill_fwd(i["q"], i["k"], i["v"], m["is_causal"])
    assert_same(o, case["outputs"]["o_golden"])
    assert_same(lse, case["outputs"]["lse"])
    assert_same(ref.mha_sdpa(i["q"], i["k"], i["v"], m["is_causal"]), case["outputs"]["o_sdpa"])


@pytest.mark.parametrize("name", names("gdn_"))
def test_oracle_gdn(name):
    case = load(name)
    i, m = case["inputs"], case["meta"]
    o, s = ref.gdn_sequential(i["q"], i["k"], i["v"], i["g"], i["beta"], i["state0"], m["scale"])
    torch.testing.assert_close(o, case["outputs"]["o"], atol=1e-6, rtol=1e-6)
    torch.testing.assert_close(s, case["outputs"]["final_state"], atol=1e-6, rtol=1e-6)


def test_oracle_gdn_bthd_layout_matches_bhtd():
    case = load("gdn_b1_h2_t48_d16_dv16")
    i, m = case["inputs"], case["meta"]
    t = lambda a: a.transpose(1, 2).contiguous()  # noqa: E731
    o, s = ref.gdn_prefill_bthd(t(i["q"]), t(i["k"]), t(i["v"]), t(i["g"]), t(i["beta"]),
                                m["scale"], i["state0"])
    torch.testing.assert_close(o.float(), t(case["outputs"]["o"]).to(o.dtype).float())
    torch.testing.assert_close(s, case["outputs"]["final_state"], atol=1e-6, rtol=1e-6)


def test_oracle_gdn_varlen_matches_batched_golden():
    """Packed sequences of equal length == the batched golden on the same tokens,
    and an empty sequence passes its initial state through."""
    case = load("gdn_b1_h2_t48_d16_dv16")
    i, m = case["inputs"], case["meta"]
    t = lambda a: a.transpose(1, 2).contiguous()  # noqa: E731  BHTD -> BTHD
    q, k, v, g, beta = (t(i[n]) for n in ("q", "k", "v", "g", "beta"))
    # two sequences of 24 tokens, an empty one between them
    cu = torch.tensor([0, 24, 24, 48])
    h0 = torch.cat([i["state0"], i["state0"] * 0.5, i["state0"] * 2.0], 0)
    o, s = ref.gdn_prefill_varlen(q, k, v, g, beta, cu, m["scale"], h0)
    split = lambda a: torch.cat([a[:, :24], a[:, 24:]], 0)  # noqa: E731
    o_b, s_b = ref.gdn_prefill_bthd(split(q), split(k), split(v), split(g), split(beta),
                                    m["scale"], torch.cat([h0[0:1], h0[2:3]], 0))
    torch.testing.assert_close(o, torch.cat([o_b[0:1], o_b[1:2]], 1), atol=0, rtol=0)
    torch.testing.assert_close(s[[0, 2]], s_b, atol=0, rtol=0)
    torch.testing.assert_close(s[1], h0[1], atol=0, rtol=0)


@pytest.mark.parametrize("name", names("gla_decode_"))
def test_oracle_gla_decode(name):
    case = load(name)
    i, m = case["inputs"], case["meta"]
    o, ns = ref.gla_decode(i["q"], i["k"], i["v"], i["gk"], i["state"], m["scale"])
    assert_same(o, case["outputs"]["o"])
    assert_same(ns, case["outputs"]["new_state"])


@pytest.mark.parametrize("name", names("ssd_chunk_scan_"))
def test_oracle_ssd_chunk_scan(name):
    case = load(name)
    i, m = case["inputs"], case["meta"]
    out = ref.ssd_chunk_scan(i["x"], i["cb"], i["dA_cumsum"], i["C"], i["prev_states"], i["dt"],
                             m["n_groups"])
    torch.testing.assert_close(out, case["outputs"]["out"], atol=1e-6, rtol=1e-5)


def test_oracle_gdn_matches_fla_naive_recurrence():
    """Second, independent pin of the GDN oracle: flash-linear-attention's own
    CPU reference (``fla.ops.gated_delta_rule.naive.naive_recurrent_gated_delta_rule``,
    fla 0.5.1 -- the ref_api the reference's GDN probe names) on the same fp32
    inputs, with an initial state and a ragged length, batch and packed forms."""
    naive = pytest.importorskip("fla.ops.gated_delta_rule.naive")
    torch.manual_seed(11)
    b, t, h, dk, dv = 2, 37, 3, 16, 8
    q = torch.nn.functional.normalize(torch.randn(b, t, h, dk), dim=-1)
    k = torch.nn.functional.normalize(torch.randn(b, t, h, dk), dim=-1)
    v = torch.randn(b, t, h, dv)
    g = torch.nn.functional.logsigmoid(torch.randn(b, t, h)) / 16
    beta = torch.sigmoid(torch.randn(b, t, h))
    h0 = torch.randn(b, h, dk, dv) * 0.1
    o, s = ref.gdn_prefill_bthd(q, k, v, g, beta, 0.3, h0)
    o_f, s_f = naive.naive_recurrent_gated_delta_rule(q, k, v, beta, g, scale=0.3,
                                                      initial_state=h0,
                                                      output_final_state=True)
    torch.testing.assert_close(o, o_f, atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(s, s_f, atol=1e-5, rtol=1e-5)
    # Packed: two sequences along the token axis, each from its own state.
    flat = lambda x: x.reshape(1, b * t, *x.shape[2:])  # noqa: E731
    cu = torch.tensor([0, t, 2 * t], dtype=torch.int32)
    o_p, s_p = ref.gdn_prefill_varlen(flat(q), flat(k), flat(v), flat(g), flat(beta), cu,
                                      0.3, h0)
    torch.testing.assert_close(o_p, flat(o_f), atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(s_p, s_f, atol=1e-5, rtol=1e-5)


def test_oracle_gla_decode_matches_fla_naive_recurrence():
    """The GLA decode oracle applied token by token equals
    flash-linear-attention's CPU reference recurrence
    (``fla.ops.gla.naive.naive_recurrent_gla``) over the same tokens: every
    step's output and the final state (fp32, fla's default scale K^-0.5)."""
    naive = pytest.importorskip("fla.ops.gla.naive")
    torch.manual_seed(12)
    b, t, h, dk, dv = 2, 9, 3, 16, 8
    q, k = torch.randn(b, t, h, dk), torch.randn(b, t, h, dk)
    v = torch.randn(b, t, h, dv)
    gk = torch.nn.functional.logsigmoid(torch.randn(b, t, h, dk))
    h0 = torch.randn(b, h, dk, dv)
    o_f, s_f = naive.naive_recurrent_gla(q, k, v, gk, initial_state=h0,
                                         output_final_state=True)
    state = h0
    for i in range(t):
        o_i, state = ref.gla_decode(q[:, i], k[:, i], v[:, i], gk[:, i], state, dk ** -0.5)
        torch.testing.assert_close(o_i, o_f[:, i], atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(state, s_f, atol=1e-5, rtol=1e-5)


def test_oracle_ssd_chunk_scan_matches_the_token_recurrence():
    """The SSD chunk-scan oracle from first principles (Mamba-2's state-space
    recurrence, per head h in group g = h // (H / G)):

        state_t = exp(dt_t A_h) state_{t-1} + dt_t x_t B_t^T     (P x N)
        y_t     = state_t C_t

    run token by token in fp64.  The chunk scan's inputs are derived from it:
    cb[l, s] = C_l . B_s, dA_cumsum = the inclusive in-chunk cumsum of dt A,
    prev_states[c] = the state entering chunk c.  Its output must equal y."""
    torch.manual_seed(13)
    b, nc, L, h, p, n, g = 2, 3, 8, 4, 4, 6, 2
    seq = nc * L
    x = torch.randn(b, seq, h, p, dtype=torch.float64)
    Bm = torch.randn(b, seq, g, n, dtype=torch.float64)
    Cm = torch.randn(b, seq, g, n, dtype=torch.float64)
    dt = torch.nn.functional.softplus(torch.randn(b, seq, h, dtype=torch.float64))
    A = -torch.rand(h, dtype=torch.float64) - 0.1
    grp = torch.arange(h) // (h // g)

    state = torch.zeros(b, h, p, n, dtype=torch.float64)
    y = torch.zeros(b, seq, h, p, dtype=torch.float64)
    prev = torch.zeros(b, nc, h, p, n, dtype=torch.float64)
    for t in range(seq):
        if t % L == 0:
            prev[:, t // L] = state
        decay = torch.exp(dt[:, t] * A)                                   # b h
        Bt, Ct = Bm[:, t][:, grp], Cm[:, t][:, grp]                       # b h n
        state = state * decay[..., None, None] + \
            (dt[:, t][..., None] * x[:, t])[..., None] * Bt[:, :, None, :]
        y[:, t] = torch.einsum("bhpn,bhn->bhp", state, Ct)

    Bc = Bm.reshape(b, nc, L, g, n)
    Cc = Cm.reshape(b, nc, L, g, n)
    cb = torch.einsum("bclgn,bcsgn->bcgls", Cc, Bc)                         # B NC G L L
    dA = torch.cumsum((dt * A).reshape(b, nc, L, h), dim=2).permute(0, 3, 1, 2)  # B H NC L
    dt_c = dt.reshape(b, nc, L, h).permute(0, 3, 1, 2)                      # B H NC L
    out = ref.ssd_chunk_scan(x.float(), cb.float(), dA.float(), Cm.float(), prev.float(),
                             dt_c.float(), g)
    torch.testing.assert_close(out.double(), y, atol=1e-4, rtol=1e-4)
