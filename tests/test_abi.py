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


def test_tp_exchange_rejects_misaligned_buffers(lib):
    # q38_tp_exchange reads part as float2 and norm_w as float4 and stores the
    # x-fragments as vectors: a pointer one of those accesses would fault on is
    # refused on the host with Q38_ERR_INVALID, before any CUDA call.
    def desc(**kw):
        d = runtime.q38_tp_exchange_desc()
        d.x_in, d.x_out, d.part, d.step = 0x1000, 0x2000, 0x3000, 0x4000
        d.region[0], d.region[1] = 0x10000, 0x20000
        d.norm_w, d.xfrag = 0x5000, 0x6000
        d.n, d.rank, d.size, d.instance, d.eps = 5120, 0, 2, 0, 1e-6
        for k, v in kw.items():
            setattr(d, k, v)
        return d

    for field, value in (("part", 0x3004), ("norm_w", 0x5008), ("xfrag", 0x6004), ("x_in", 0x1002),
                         ("x_out", 0x2001), ("step", 0x4002)):
        rc = lib.q38_tp_exchange(C.byref(desc(**{field: value})), None)
        assert rc == 1, field
        assert b"misaligned" in lib.q38_last_error(), field
    rc = lib.q38_tp_exchange(C.byref(desc(instance=511)), None)
    assert rc == 1 and b"instance <= 510" in lib.q38_last_error()
