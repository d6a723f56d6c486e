"""The no-allocation Gated DeltaNet entry point (collected last on purpose).

tileops_gdn_prefill_fwd_noalloc serves callers that cannot allocate device
memory at call time (a call recorded into a CUDA graph, or a host runtime /
plugin with no device allocator): it keeps the per-chunk scratch in a fixed
16 MiB array inside the library instead of a caller workspace.  This test
calls it through the C ABI twice in a row, on different inputs (the array
keeps the previous call's contents, which must not leak into the next
result), checks each result against the oracle's sequential GDN recurrence
within the GDN tests' tolerances and bit-for-bit against the workspace entry
point tileops_gdn_prefill_fwd (the same kernels on the same inputs); it also
checks that a shape needing more than the fixed scratch is refused.
"""

import ctypes

import pytest
import torch

from oracle import reference as ref
from tileops import _native
from tileops.workloads.linear_attention import GdnPrefillWorkload

pytestmark = pytest.mark.gpu

# The GDN tests' tolerances against the oracle: the bf16 output o and the
# fp32 final state (measured bound with a 2x margin; see test_gated_delta_net).
TOL = dict(atol=1e-2, rtol=1e-2)
STATE_TOL = dict(atol=8e-3, rtol=1e-3)
BF16 = 2


def _args(q, k, v, g, beta, h0, o, hT):
    p = _native.ptr
    return (p(q), p(k), p(v), p(g), p(beta), p(h0), p(o), p(hT))


def _shape_args(q, v):
    b, t, h, dk = q.shape
    return (b, t, h, dk, v.shape[-1], 64, float(dk**-0.5), BF16)


def _with_workspace(q, k, v, g, beta, h0):
    lib = _native.lib()
    b, t, h, dk = q.shape
    o = torch.empty(b, t, h, v.shape[-1], dtype=torch.bfloat16, device="cuda")
    hT = torch.empty(b, h, dk, v.shape[-1], dtype=torch.float32, device="cuda")
    ws = torch.empty(lib.tileops_gdn_workspace_bytes(b, t, h, dk, v.shape[-1]),
                     dtype=torch.uint8, device="cuda")
    rc = lib.tileops_gdn_prefill_fwd(*_args(q, k, v, g, beta, h0, o, hT), _native.ptr(ws),
                                     *_shape_args(q, v), _native.stream_handle(q.device))
    assert rc == 0, rc
    return o, hT


def _no_alloc(q, k, v, g, beta, h0):
    lib = _native.lib()
    b, t, h, dk = q.shape
    o = torch.empty(b, t, h, v.shape[-1], dtype=torch.bfloat16, device="cuda")
    hT = torch.empty(b, h, dk, v.shape[-1], dtype=torch.float32, device="cuda")
    rc = lib.tileops_gdn_prefill_fwd_noalloc(*_args(q, k, v, g, beta, h0, o, hT),
                                             *_shape_args(q, v), _native.stream_handle(q.device))
    assert rc == 0, rc
    return o, hT


def test_no_alloc_entry_point_matches_workspace_entry_point():
    cases = [GdnPrefillWorkload(2, 384, 2, 128, 128).gen_inputs(),
             GdnPrefillWorkload(1, 1000, 3, 128, 128).gen_inputs()]
    h0 = torch.randn(1, 3, 128, 128, device="cuda") * 0.1
    for i, (q, k, v, g, beta) in enumerate(cases):  # two calls in a row
        init = h0 if i == 1 else None
        o_ref, s_ref = _with_workspace(q, k, v, g, beta, init)
        o, s = _no_alloc(q, k, v, g, beta, init)
        torch.cuda.synchronize()
        assert torch.equal(o, o_ref) and torch.equal(s, s_ref)
        o_gold, s_gold = ref.gdn_prefill_bthd(q, k, v, g, beta, None, init)
        torch.testing.assert_close(o.cpu().float(), o_gold.float(), **TOL)
        torch.testing.assert_close(s.cpu(), s_gold, **STATE_TOL)


def test_no_alloc_rejects_shapes_beyond_its_scratch():
    lib = _native.lib()
    null = ctypes.c_void_p(0)
    # 1 * 8 heads * 64 chunks of 64 tokens = 512 chunks > 404 that fit in 16 MiB
    assert lib.tileops_gdn_workspace_bytes(1, 4096, 8, 128, 128) > 16 << 20
    rc = lib.tileops_gdn_prefill_fwd_noalloc(*([null] * 8), 1, 4096, 8, 128, 128, 64, 0.1, BF16,
                                             null)
    assert rc == _native.EBADSHAPE
