"""CPU tests of the C ABI boundary: the library loads without a GPU, exports
exactly what include/ovb200.h declares, and rejects bad arguments before
touching the device (the reference's contract, ov_gemm.h / gemm.cpp)."""
from __future__ import annotations

import ctypes as C
import re
import subprocess

import pytest

from ovnative_b200 import _lib as L


def header_functions() -> set[str]:
    src = open(L.HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return set(re.findall(r"\b(ovb_\w+)\s*\(", src))


def test_library_loads_and_exports_header():
    lib = L.lib()
    declared = header_functions()
    assert declared, "no functions parsed from the header"
    for name in declared:
        assert hasattr(lib, name), f"{name} declared in ovb200.h but not exported"
    out = subprocess.run(["nm", "-D", "--defined-only", L.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\sT\s(ovb_\w+)$", out, flags=re.M))
    assert exported == declared
    assert set(L.SIGNATURES) == declared


def test_abi_version_and_sizes():
    lib = L.lib()
    assert lib.ovb_abi_version() == 1
    # s8_nk_quant_bytes / s8_nk_quant_scales (gemm.cpp:623-631)
    assert lib.ovb_quant_bytes(7, 69) == 7 * 96
    assert lib.ovb_quant_scales(7, 69) == 7 * 3
    assert lib.ovb_quant_bytes(0, 69) == 0
    assert lib.ovb_linear_workspace_bytes(256, 1024) == 256 * 1024 + 256 * 32 * 4


def test_noop_and_argument_errors_without_device():
    lib = L.lib()
    # M <= 0: silent no-op (gemm.cpp:761)
    assert lib.ovb_linear_q(0, None, None, None, None, 0, 0, None) == L.OVB_OK
    assert lib.ovb_quantize(5, 0, None, 0, None, None, 0, None) == L.OVB_OK
    # null weight handle -> invalid argument with a message
    assert lib.ovb_linear_q(4, None, None, None, None, 0, 0, None) == L.OVB_ERR_INVALID_ARG
    assert b"null" in lib.ovb_last_error()
    out = C.c_void_p()
    assert lib.ovb_weight_create(None, 0, 0, 16, None, 0, None, C.byref(out)) == \
        L.OVB_ERR_INVALID_ARG
    assert lib.ovb_weight_create(None, 7, 8, 16, None, 0, None, C.byref(out)) == \
        L.OVB_ERR_INVALID_ARG
    with pytest.raises(ValueError):
        L.check(L.OVB_ERR_INVALID_ARG)


def test_static_linear_checks_arguments_before_the_device():
    """ovb_linear_static rejects a null weight and null A/C before it looks
    up its device array or enqueues anything (no GPU here)."""
    lib = L.lib()
    assert lib.ovb_linear_static(0, None, None, 0, None, 0, 0, None) == L.OVB_OK
    assert lib.ovb_linear_static(4, None, None, 0, None, 0, 0, None) == L.OVB_ERR_INVALID_ARG
    assert b"null" in lib.ovb_last_error()
    # A non-null handle is not read before the A/C check.
    fake = C.create_string_buffer(4096)
    assert lib.ovb_linear_static(4, C.addressof(fake), None, 0, None, 0, 0, None) == \
        L.OVB_ERR_INVALID_ARG
    assert b"A/C" in lib.ovb_last_error()


def test_rope_entry_points_check_arguments_before_the_device():
    """The RoPE table, the unfused q/k norm + RoPE and the fused q|k|v GEMM
    reject bad shapes and null pointers without touching a device; zero rows
    are a no-op."""
    lib = L.lib()
    assert lib.ovb_rope_table(None, 0, 128, 1e6, None, None) == L.OVB_OK
    assert lib.ovb_rope_table(None, 4, 64, 1e6, None, None) == L.OVB_ERR_INVALID_ARG
    assert b"head_dim" in lib.ovb_last_error()
    assert lib.ovb_rope_table(None, 4, 128, 1e6, None, None) == L.OVB_ERR_INVALID_ARG
    assert lib.ovb_qk_norm_rope_f16(0, None, None, None, 16, 8, 128, None, None, 1e-6, None,
                                    None, None, None, None) == L.OVB_OK
    assert lib.ovb_qk_norm_rope_f16(4, None, None, None, 16, 8, 128, None, None, 1e-6, None,
                                    None, None, None, None) == L.OVB_ERR_INVALID_ARG
    assert lib.ovb_qk_norm_rope_f16(4, None, None, None, 16, 8, 96, None, None, 1e-6, None,
                                    None, None, None, None) == L.OVB_ERR_INVALID_ARG
    assert b"head_dim" in lib.ovb_last_error()
    assert lib.ovb_linear_h_qk_rope(0, None, None, 16, 8, 128, None, None, 1e-6, None, None,
                                    None, None, None) == L.OVB_OK
    assert lib.ovb_linear_h_qk_rope(4, None, None, 16, 8, 128, None, None, 1e-6, None, None,
                                    None, None, None) == L.OVB_ERR_INVALID_ARG
    assert b"null" in lib.ovb_last_error()


def test_batched_sampler_checks_arguments_before_the_device():
    """ovb_guided_sample_batch: zero pairs are a no-op; too many pairs, null
    buffers and lengths shorter than the target are refused on the host."""
    lib = L.lib()
    assert lib.ovb_guided_sample_batch(0, None, 8, 1025, 2.0, 5.0, 1024, None, None,
                                       None) == L.OVB_OK
    assert lib.ovb_guided_sample_batch(65, None, 8, 1025, 2.0, 5.0, 1024, None, None,
                                       None) == L.OVB_ERR_INVALID_ARG
    pred = C.create_string_buffer(64)
    pairs = (L.GuidedPair * 1)(L.GuidedPair(None, 10, None, 10, 5))
    assert lib.ovb_guided_sample_batch(1, pairs, 8, 1025, 2.0, 5.0, 1024, C.addressof(pred),
                                       C.addressof(pred), None) == L.OVB_ERR_INVALID_ARG
    assert b"null" in lib.ovb_last_error()
    buf = C.create_string_buffer(64)
    pairs = (L.GuidedPair * 1)(L.GuidedPair(C.addressof(buf), 4, C.addressof(buf), 10, 5))
    assert lib.ovb_guided_sample_batch(1, pairs, 8, 1025, 2.0, 5.0, 1024, C.addressof(pred),
                                       C.addressof(pred), None) == L.OVB_ERR_INVALID_ARG
    assert b"target_len" in lib.ovb_last_error()
