"""The C-ABI library builds, loads without a GPU and exports every function
that include/q38rt.h declares.  No compute call is made here."""
from __future__ import annotations

import ctypes as C

import pytest

from qwen382743090_b200 import build, runtime


@pytest.fixture(scope="module")
def lib():
    build.build()
    return runtime.lib()


def test_header_declares_core_entry_points():
    names = set(runtime.header_functions())
    for must in ("q38_ctx_open", "q38_ctx_close", "q38_alloc", "q38_free", "q38_memcpy_h2d", "q38_memcpy_d2h",
                 "q38_gemv_packed", "q38_q5k_sm86_soa_gemv_vec", "q38_last_error"):
        assert must in names


def test_library_exports_every_declared_symbol(lib):
    missing = [n for n in runtime.header_functions() if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_version_string(lib):
    assert b"sm_100a" in lib.q38_version()


def test_argument_validation_needs_no_gpu(lib):
    # shape errors are rejected on the host before any CUDA call
    rc = lib.q38_q5k_sm86_soa_gemv_vec(16, 16, 16, 16, 16, 300, 8, None)
    assert rc == 1
    assert b"multiple of 256" in lib.q38_last_error()
    rc = lib.q38_q5k_sm86_soa_gemv_vec(16, 16, 24, 16, 16, 1024, 8, None)
    assert rc == 1 and b"aligned" in lib.q38_last_error()
    assert lib.q38_xpack_bytes(2, 1024, 1) == 0
    assert lib.q38_xpack_bytes(3, 1024, 1) > 3 * 1024


def test_no_device_is_an_error_not_a_fallback(lib):
    if runtime.device_count() > 0:
        pytest.skip("a GPU is visible")
    h = C.c_void_p()
    rc = lib.q38_ctx_open(0, C.byref(h))
    assert rc != 0
