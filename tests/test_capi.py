"""The C ABI shared library without a GPU: it loads, exports exactly what include/cppinf_b200.h declares, validates
arguments on the host with the reference's messages and status codes before touching CUDA, and builds the RoPE
angle table on the host bit-identically to the oracle (and so to the reference's rope.cpp)."""

from __future__ import annotations

import ctypes
import subprocess

import numpy as np
import pytest

from cppinf_b200 import capi


@pytest.fixture(scope="module")
def lib():
    return capi.load()


def test_library_exports_every_declared_symbol(lib):
    declared = capi.header_symbols()
    assert len(declared) >= 19
    for name in declared:
        assert hasattr(lib, name), name
    exported = subprocess.run(["nm", "-D", "--defined-only", str(capi.LIB_PATH)], capture_output=True, text=True,
                              check=True).stdout
    exported_names = {line.split()[-1] for line in exported.splitlines() if " T " in line}
    assert exported_names == set(declared), "the library must export the C ABI and nothing else"


def test_abi_version_and_status_names(lib):
    assert lib.cppinf_abi_version() == 1
    assert lib.cppinf_status_name(capi.ERR_OVERFLOW) == b"CPPINF_ERR_OVERFLOW"


def _status(lib, name, *args):
    return getattr(lib, name)(*args)


def test_rms_norm_validation_messages(lib):
    assert _status(lib, "cppinf_rms_norm", 0, None, 4, None, None, 2, 4, -1.0, None) == capi.ERR_INVALID_ARGUMENT
    assert capi.last_error() == "rms_norm requires a non-negative epsilon."
    assert _status(lib, "cppinf_rms_norm", 0, None, 0, None, None, 2, 0, 1e-6, None) == capi.ERR_INVALID_ARGUMENT
    assert capi.last_error() == "rms_norm requires a non-empty last dimension."
    assert _status(lib, "cppinf_rms_norm", 5, None, 4, None, None, 2, 4, 1e-6, None) == capi.ERR_INVALID_ARGUMENT
    assert "unsupported dtype" in capi.last_error()
    assert _status(lib, "cppinf_rms_norm", 0, None, 4, None, None, 2, 4, 1e-6, None) == capi.ERR_INVALID_ARGUMENT
    assert "null pointer" in capi.last_error()
    # zero rows is a valid empty op: no CUDA call, success
    assert _status(lib, "cppinf_rms_norm", 0, None, 4, None, None, 0, 4, 1e-6, None) == capi.OK


def test_softmax_validation_messages(lib):
    assert _status(lib, "cppinf_scaled_causal_softmax_f32", None, None, 1, 2, 3, 1.0, None) == \
        capi.ERR_INVALID_ARGUMENT
    assert capi.last_error() == "scaled_causal_softmax_last_dim requires square attention score matrices."
    assert _status(lib, "cppinf_scaled_causal_softmax_f32", None, None, 1, 2, 2, float("nan"), None) == \
        capi.ERR_INVALID_ARGUMENT
    assert capi.last_error() == "scaled_causal_softmax_last_dim requires a finite scale."
    offs = capi.i64_array([0] * 65)
    assert _status(lib, "cppinf_scaled_position_causal_softmax_f32", None, None, 65, 1, 2, 2, 1.0, offs, offs, offs,
                   None) == capi.ERR_UNSUPPORTED
    bad = capi.i64_array([5])
    ok = capi.i64_array([2])
    assert _status(lib, "cppinf_scaled_position_causal_softmax_f32", None, None, 1, 1, 2, 2, 1.0, ok, bad, ok,
                   None) == capi.ERR_INVALID_ARGUMENT
    assert "exceeds the padded sequence capacity" in capi.last_error()


def test_argmax_and_rope_validation(lib):
    assert _status(lib, "cppinf_row_argmax", 0, None, 1, 1 << 31, 1 << 31, None, None) == capi.ERR_OVERFLOW
    assert _status(lib, "cppinf_row_argmax", 0, None, 1, 0, 0, None, None) == capi.ERR_INVALID_ARGUMENT
    assert _status(lib, "cppinf_rope", 0, None, 1, 2, 3, 6, 3, 1, 1, 0, None, 8, None, None) == \
        capi.ERR_INVALID_ARGUMENT
    assert capi.last_error() == "apply_rope requires an even head size."
    assert _status(lib, "cppinf_rope", 0, None, 1, 2, 4, 8, 4, 1, 2, 0, None, 8, None, None) == \
        capi.ERR_INVALID_ARGUMENT
    assert capi.last_error() == "apply_rope requires the sequence dimension to be 0 or 1."
    assert _status(lib, "cppinf_rope", 0, None, 1, 9, 4, 36, 4, 1, 1, 0, None, 8, None, None) == \
        capi.ERR_OUT_OF_RANGE
    # head_dim 100 has no fused kernel (100 / 8 is not a power of two): the caller composes rms_norm + rope instead
    assert _status(lib, "cppinf_qk_norm_rope", 0, None, None, None, None, None, None, 4, 2, 1, 100, 0, 1e-6, None,
                   16, None) == capi.ERR_UNSUPPORTED
    assert _status(lib, "cppinf_qk_norm_rope", 0, None, None, None, None, None, None, 4, 2, 1, 128, 10, 1e-6, None,
                   13, None) == capi.ERR_OUT_OF_RANGE


def test_check_maps_status_to_reference_exception_types(lib):
    with pytest.raises(ValueError, match="non-negative epsilon"):
        capi.check(_status(lib, "cppinf_rms_norm", 0, None, 4, None, None, 2, 4, -1.0, None))
    with pytest.raises(OverflowError):
        capi.check(_status(lib, "cppinf_row_argmax", 0, None, 1, 1 << 31, 1 << 31, None, None))
    with pytest.raises(IndexError):
        capi.check(_status(lib, "cppinf_rope", 0, None, 1, 9, 4, 36, 4, 1, 1, 0, None, 8, None, None))
    with pytest.raises(NotImplementedError):
        capi.check(_status(lib, "cppinf_qk_norm_rope", 0, None, None, None, None, None, None, 4, 2, 1, 100, 0, 1e-6,
                           None, 16, None))


@pytest.mark.parametrize("base,head_dim,positions", [(1e6, 128, 2048), (10000.0, 64, 300), (500000.0, 256, 17)])
def test_host_rope_table_is_bit_identical_to_oracle(oracle, base, head_dim, positions):
    table = capi.rope_table(base, head_dim, positions)
    assert np.array_equal(table, oracle.rope_table(base, head_dim, positions))


def test_host_rope_table_validation(lib):
    out = (ctypes.c_float * 8)()
    assert _status(lib, "cppinf_rope_table", -1.0, 8, 1, out) == capi.ERR_INVALID_ARGUMENT
    assert capi.last_error() == "apply_rope requires a positive finite rope base."
    assert _status(lib, "cppinf_rope_table", 1e6, 7, 1, out) == capi.ERR_INVALID_ARGUMENT
