"""A bounded device-side wait that runs out, on the GPU, without faulting it.

Every tensor-core kernel of the library (attention, GDN, SSD chunk scan,
dense conv1d) has the same give-up path: when a wait runs out it records
device error 1, lets its own copies land, frees TMEM and returns, so the
context stays usable.  ``tileops_selftest_wait_timeout`` runs that path on
purpose: it waits ~1 ms, polling, on an mbarrier nothing arrives on while
holding TMEM and a bulk copy in flight.  The test checks what the host sees
afterwards: the status word, the drained copy, the time the wait took, that
the flag clears, and that a tensor-core op launched next runs clean.
"""

import ctypes

import pytest
import torch

from tileops import _native
from tileops.ops.attention import MultiHeadAttentionFwdOp

pytestmark = pytest.mark.gpu


def _run_selftest(nbytes: int, limit_ns: int):
    dev = torch.device("cuda", 0)
    src = (torch.arange(nbytes, device=dev) % 251).to(torch.uint8)
    out = torch.zeros(6, dtype=torch.int32, device=dev)
    stream = _native.stream_handle(dev)
    status = _native.lib().tileops_selftest_wait_timeout(
        ctypes.c_void_p(src.data_ptr()), nbytes, limit_ns, ctypes.c_void_p(out.data_ptr()), stream)
    assert status == _native.OK
    torch.cuda.synchronize(dev)
    return src, out, stream


def test_wait_runs_out_reports_and_recovers():
    stream = _native.stream_handle(torch.device("cuda", 0))
    _native.lib().tileops_device_error_flag(stream, 1)  # start from a clear word
    src, out, stream = _run_selftest(4096, 1_000_000)  # 1 ms limit
    got = out.cpu().tolist()
    assert got[0] == 1, "the unarmed wait did not give up"
    assert got[1] == 1, "the drain did not see the in-flight copy land"
    assert got[2] == int(src.to(torch.int64).sum()), "copied bytes read before they landed"
    assert got[3] == 1, "TMEM was not released"
    waited_ns = (got[5] << 32) | (got[4] & 0xffffffff)
    # It gave up once the limit had passed, and not much later: the polls are
    # 64 ns apart and the timer is read after each one.
    assert 1_000_000 <= waited_ns < 50_000_000, waited_ns
    # The host sees the timeout code once, and reading with clear resets it.
    assert _native.lib().tileops_device_error_flag(stream, 1) == 1
    assert _native.lib().tileops_device_error_flag(stream, 0) == 0
    # The context is still usable: a real tensor-core op runs and sets no flag.
    q, k, v = (torch.randn(1, 256, 2, 128, device="cuda", dtype=torch.bfloat16)
               for _ in range(3))
    o, lse = MultiHeadAttentionFwdOp(1, 2, 256, 128, False, torch.bfloat16)(q, k, v)
    torch.cuda.synchronize()
    assert torch.isfinite(o.float()).all() and torch.isfinite(lse).all()
    assert _native.lib().tileops_device_error_flag(stream, 1) == 0


def test_two_timeouts_in_a_row():
    stream = _native.stream_handle(torch.device("cuda", 0))
    _native.lib().tileops_device_error_flag(stream, 1)
    _, out1, stream = _run_selftest(256, 200_000)
    _, out2, _ = _run_selftest(16, 200_000)
    assert out1[0].item() == 1 and out2[0].item() == 1
    assert _native.lib().tileops_device_error_flag(stream, 1) == 1
    assert _native.lib().tileops_device_error_flag(stream, 1) == 0


def test_selftest_rejects_bad_arguments():
    dev = torch.device("cuda", 0)
    src = torch.zeros(8192, dtype=torch.uint8, device=dev)
    out = torch.zeros(6, dtype=torch.int32, device=dev)
    stream = _native.stream_handle(dev)
    f = _native.lib().tileops_selftest_wait_timeout
    p, o = ctypes.c_void_p(src.data_ptr()), ctypes.c_void_p(out.data_ptr())
    assert f(p, 8192, 1_000_000, o, stream) == _native.EBADSHAPE  # over 4096 bytes
    assert f(p, 24, 1_000_000, o, stream) == _native.EBADSHAPE  # not a multiple of 16
    assert f(p, 64, 10, o, stream) == _native.EBADSHAPE  # limit below 1 us
    assert f(ctypes.c_void_p(src.data_ptr() + 8), 64, 1_000_000, o, stream) == _native.EALIGN
    assert f(None, 64, 1_000_000, o, stream) == _native.EINVAL
    torch.cuda.synchronize()
    assert out.sum().item() == 0  # nothing was launched
