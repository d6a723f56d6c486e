"""The C-ABI library: it loads, exports every function the header declares,
and rejects invalid arguments on the host before touching the GPU.  CPU only
(every call here fails argument validation before any CUDA call)."""

import ctypes

import pytest

from tileops import _native

NULL = ctypes.c_void_p(0)


def test_library_loads():
    assert _native.LIB_PATH.exists(), "run __graft_entry__.build() first"
    assert _native.lib().tileops_abi_version() == 1


def test_every_declared_entry_point_is_exported():
    declared = _native.declared_entry_points()
    assert len(declared) >= 19
    handle = _native.lib()
    missing = [name for name in declared if not hasattr(handle, name)]
    assert not missing, f"declared in include/tileops_c.h but not exported: {missing}"


def test_every_declared_entry_point_has_a_python_signature():
    assert set(_native.declared_entry_points()) <= set(_native._SIGNATURES)


def test_status_strings():
    lib = _native.lib()
    for code in (0, -1, -2, -3, -4, -5, -6):
        assert lib.tileops_status_string(code)
    assert lib.tileops_status_string(0) == b"ok"
    assert lib.tileops_status_string(-99) == b"unknown status"


@pytest.mark.parametrize(
    "name",
    ["tileops_hardswish_fwd", "tileops_hardsigmoid_fwd", "tileops_isnan_fwd",
     "tileops_isinf_fwd", "tileops_isfinite_fwd", "tileops_bitwise_not_fwd"],
)
def test_unary_rejects_negative_size(name):
    assert getattr(_native.lib(), name)(NULL, NULL, -1, 0, NULL) == _native.EBADSHAPE


@pytest.mark.parametrize("name", ["tileops_hardswish_fwd", "tileops_isnan_fwd"])
def test_unary_empty_is_ok_and_null_is_rejected(name):
    lib = _native.lib()
    assert getattr(lib, name)(NULL, NULL, 0, 0, NULL) == _native.OK
    assert getattr(lib, name)(NULL, NULL, 16, 0, NULL) == _native.EINVAL


def test_bitwise_not_rejects_float_dtype():
    assert _native.lib().tileops_bitwise_not_fwd(NULL, NULL, 16, 0, NULL) == _native.EBADDTYPE


def test_clamp_requires_a_bound():
    r = _native.lib().tileops_clamp_scalar_fwd(NULL, NULL, 16, 0, 0, 0.0, 0, 0.0, NULL)
    assert r == _native.EINVAL


def test_gated_and_norm_reject_bad_shapes():
    lib = _native.lib()
    assert lib.tileops_gelu_and_mul_fwd(NULL, NULL, -1, 8, 2, NULL) == _native.EBADSHAPE
    assert lib.tileops_gelu_tanh_and_mul_fwd(NULL, NULL, 4, -8, 2, NULL) == _native.EBADSHAPE
    assert lib.tileops_fused_add_layer_norm_fwd(
        NULL, NULL, NULL, NULL, NULL, NULL, 4, 0, 1e-5, 2, 2, NULL) == _native.EBADSHAPE
    assert lib.tileops_fused_add_layer_norm_fwd(
        NULL, NULL, NULL, NULL, NULL, NULL, 4, 8, 1e-5, 2, 2, NULL) == _native.EINVAL


def test_conv_rejects_bad_geometry():
    lib = _native.lib()
    args = [NULL] * 4
    # k = 0
    assert lib.tileops_conv1d_depthwise_fwd(*args, 1, 4, 16, 16, 0, 1, 0, 1, 2, 2, 0,
                                            NULL) == _native.EBADSHAPE
    # unknown activation
    assert lib.tileops_conv1d_depthwise_fwd(*args, 1, 4, 16, 16, 3, 1, 1, 1, 2, 2, 7,
                                            NULL) == _native.EINVAL
    # c_in not divisible by groups
    assert lib.tileops_conv1d_direct_fwd(*args, 1, 6, 16, 8, 16, 3, 1, 1, 1, 4, 1,
                                         NULL) == _native.EBADSHAPE


def test_status_maps_to_python_exceptions():
    with pytest.raises(ValueError, match="invalid shape"):
        _native.call("tileops_hardswish_fwd", NULL, NULL, -5, 0, NULL)
    with pytest.raises(_native.NativeLibraryError):
        _native.call("tileops_no_such_entry")


def test_gdn_varlen_workspace_and_validation():
    lib = _native.lib()
    per = (64 * 128 + 64 * 128 + 64 * 64) * 2 + (2 * 64 + 4) * 4
    # (total / 64 + N) chunk slots per head, then the int32 slot table (16-byte rounded)
    slots = 1000 // 64 + 3
    assert lib.tileops_gdn_varlen_workspace_bytes(1000, 3, 2, 128, 128) == (
        2 * slots * per + (slots * 4 + 15) // 16 * 16)
    assert lib.tileops_gdn_varlen_workspace_bytes(64, 1, 1, 96, 128) == -1
    assert lib.tileops_gdn_varlen_workspace_bytes(-1, 1, 1, 128, 128) == -1
    fn = lib.tileops_gdn_prefill_varlen_fwd
    head = [NULL] * 5 + [NULL]  # q, k, v, g, beta, cu_seqlens
    tail = [NULL] * 4           # initial_state, o, final_state, workspace
    # no sequences: nothing to do
    assert fn(*head, 0, *tail, 0, 2, 128, 128, 64, 0.1, 0, 2, NULL) == _native.OK
    assert fn(*head, 2, *tail, 128, 2, 128, 128, 32, 0.1, 0, 2, NULL) == _native.EBADSHAPE
    assert fn(*head, 2, *tail, 128, 2, 128, 128, 64, 0.1, 0, 1, NULL) == _native.EBADDTYPE
    assert fn(*head, 2, *tail, 128, 2, 96, 128, 64, 0.1, 0, 2, NULL) == _native.EBADSHAPE
    assert fn(*head, -1, *tail, 128, 2, 128, 128, 64, 0.1, 0, 2, NULL) == _native.EBADSHAPE
    # unknown flag bits
    assert fn(*head, 2, *tail, 128, 2, 128, 128, 64, 0.1, 4, 2, NULL) == _native.EINVAL
    # cu_seqlens NULL: total_len must split evenly into num_seqs sequences
    assert fn(*head, 3, *tail, 128, 2, 128, 128, 64, 0.1, 0, 2, NULL) == _native.EBADSHAPE
    # NULL tensors
    assert fn(*head, 2, *tail, 128, 2, 128, 128, 64, 0.1, 1, 2, NULL) == _native.EINVAL


def test_gdn_workspace_and_validation():
    lib = _native.lib()
    assert lib.tileops_gdn_workspace_bytes(4, 8192, 16, 128, 128) == 4 * 16 * 128 * (
        (64 * 128 + 64 * 128 + 64 * 64) * 2 + (2 * 64 + 4) * 4)
    assert lib.tileops_gdn_workspace_bytes(1, 64, 1, 96, 128) == -1
    args = [NULL] * 9
    # chunk size other than 64
    assert lib.tileops_gdn_prefill_fwd(*args, 1, 64, 1, 128, 128, 32, 0.1, 2, NULL) == (
        _native.EBADSHAPE)
    # fp16 is not supported
    assert lib.tileops_gdn_prefill_fwd(*args, 1, 64, 1, 128, 128, 64, 0.1, 1, NULL) == (
        _native.EBADDTYPE)
    # NULL pointers
    assert lib.tileops_gdn_prefill_fwd(*args, 1, 64, 1, 128, 128, 64, 0.1, 2, NULL) == (
        _native.EINVAL)


def test_mha_validation():
    lib = _native.lib()
    args = [NULL] * 5
    assert lib.tileops_mha_fwd(*args, 1, 4, 3, 64, 64, 128, 0, 0.1, 2, NULL) == _native.EBADSHAPE
    assert lib.tileops_mha_fwd(*args, 1, 4, 4, 64, 64, 96, 0, 0.1, 2, NULL) == _native.EBADSHAPE
    assert lib.tileops_mha_fwd(*args, 1, 4, 4, 64, 64, 128, 0, 0.1, 0, NULL) == _native.EBADDTYPE
    assert lib.tileops_mha_fwd(*args, 1, 4, 4, 128, 64, 128, 1, 0.1, 2, NULL) == (
        _native.EBADSHAPE)
    # More CTAs than a 32-bit linear block index can number (64 x 1023 heads
    # x 2^22 query-tile pairs) is refused, not launched.
    assert lib.tileops_mha_fwd(*args, 64, 1023, 1023, 1 << 30, 1 << 30, 128, 0, 0.1, 2,
                               NULL) == _native.EBADSHAPE
    # Batch x heads above the grid's y limit.
    assert lib.tileops_mha_fwd(*args, 2, 32768, 32768, 64, 64, 128, 0, 0.1, 2, NULL) == (
        _native.EBADSHAPE)
